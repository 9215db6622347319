// graph_canon.h -- Reshape, Sub, Slice and Concat nodes restated as the
// affine kinds the level schedule takes.
//
// Luna bounds these nodes on their own (BoundedReshapeNode.cpp:40-130,
// BoundedSubNode.cpp:61-240, BoundedSliceNode.cpp:113-201,
// BoundedConcatNode.cpp:56-220).  Each is an affine map with a fixed 0/±1
// structure, so it folds exactly into the affine node next to it: the folded
// node computes the same interval and linear bounds, with only the fp32
// order of a few additions changed.  The rewrites:
//   RESHAPE            -> FLATTEN (Luna's Reshape flattens, OnnxToTorch.cpp:1959)
//   SUB on the input   -> an input transform x' = x - c or c - x, applied to
//                         the boxes before anything else (IBP of Luna's Sub,
//                         the same fp32 subtraction)
//   SUB on LINEAR/CONV -> that node with bias b - c (or weight -W, bias c - b)
//   SLICE of a LINEAR  -> that LINEAR with the selected rows
//   SLICE into LINEARs -> those LINEARs with zero columns for the features
//                         the slice drops, reading the slice's producer
//   CONCAT of LINEARs / CONVs of one producer -> one node with the rows /
//                         output channels stacked in operand order
// Nodes a rewrite leaves without a path to the output are marked dead; node
// ids do not change, so intermediate bounds stay keyed by Luna's node ids.
#pragma once

#include "luna_b200.h"

#include <memory>
#include <string>
#include <vector>

namespace lb200 {

struct CanonGraph {
    std::vector<lb200_node_desc> nodes;
    std::vector<std::unique_ptr<std::vector<float>>> store;  // arrays of rewritten nodes
    std::vector<char> dead;
    lb200_graph_desc desc{};
    // Sub on the input node: x' = x - in_const (in_neg = false) or
    // in_const - x (in_neg = true), per feature in Luna's flat order.
    bool in_tf = false;
    bool in_neg = false;
    std::vector<float> in_const;
};

// Throws std::invalid_argument naming the node when a node of these kinds
// sits where no exact rewrite exists.
CanonGraph canonicalize(const lb200_graph_desc* g);

}  // namespace lb200
