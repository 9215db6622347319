// luna_b200_shim.h -- the Luna-side adapter of the B200 engine.
//
// This is the code a Luna maintainer adds to Luna's tree to route
// TorchModel::compute_bounds to the engine.  It is compiled against Luna's
// headers and LibTorch (oracle/Makefile builds it from the reference tree),
// and reaches the engine only through the C ABI in include/luna_b200.h: no
// torch::Tensor crosses into the engine, and the engine never sees Luna's
// classes.
//
// The classes mirror Luna's interface names and constructor arguments:
//   lb200_luna::Bounded*Node   <- NLR::Bounded*Node constructors
//                                 (src/engine/nodes/BoundedLinearNode.h:21-22,
//                                  BoundedConvNode.h:27-29,
//                                  BoundedConvTransposeNode.h:23-25,
//                                  BoundedBatchNormNode.h:23-30, ...)
//   lb200_luna::TorchModel     <- NLR::TorchModel(nodes, inputIndices,
//                                 outputIndex, dependencies)
//                                 (src/engine/TorchModel.h:47-50) with
//                                 setInputBounds / setSpecificationMatrix /
//                                 compute_bounds / runCROWN / runAlphaCROWN /
//                                 getFinalAnalysisBounds (:77-110).
// A front end that builds Luna nodes (OnnxToTorchParser) builds the shim's
// nodes from the same torch modules and tensors at the same place: Luna's
// nodes keep their modules private, so the shim takes what their
// constructors take rather than reading a finished NLR::TorchModel.
//
// Results follow TorchModel::compute_bounds (TorchModel.cpp:653-698): the
// LunaConfiguration flags in force at the call (ALPHA_*, OPTIMIZE_*,
// STOP_*_ON_VERIFIED, ENABLE_FIRST_LINEAR_IBP, USE_PATCHES_MODE, ...) are
// passed to the engine as lb200_options.  Errors raise std::runtime_error
// carrying lb200_last_error(), as Luna reports failures by exception.
#pragma once

#include "../include/luna_b200.h"

#include "BoundedTensor.h"
#include "configuration/LunaConfiguration.h"
#include "conv/ConvolutionMode.h"
#include "nodes/BoundedTorchNode.h"

#include <torch/torch.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace lb200_luna {

// One node: the engine's description plus the host copies of its tensors.
class BoundedNode {
public:
    virtual ~BoundedNode() = default;
    NLR::NodeType getNodeType() const { return static_cast<NLR::NodeType>(d_.type); }
    // Output shape as Luna's conv nodes take it ({1, C, H, W}); flat nodes
    // take setOutputSize (BoundedTorchNode::setOutputSize).
    void setOutputShape(const std::vector<int>& shape);
    void setOutputSize(unsigned size);
    unsigned getOutputSize() const;
    const lb200_node_desc& desc() const { return d_; }
    const std::vector<float>& weights() const { return w_; }
    const std::vector<float>& biases() const { return b_; }
    const std::vector<float>& means() const { return mean_; }
    const std::vector<float>& vars() const { return var_; }
    const std::vector<float>& constants() const { return const_; }

protected:
    explicit BoundedNode(NLR::NodeType t);
    void keep(const torch::Tensor& t, std::vector<float>& dst);
    lb200_node_desc d_{};
    std::vector<float> w_, b_, mean_, var_, const_;
};

class BoundedInputNode : public BoundedNode {
public:
    BoundedInputNode(unsigned inputIndex, unsigned inputSize, const std::string& name = "");
};

class BoundedLinearNode : public BoundedNode {
public:
    // alpha: ONNX Gemm scale, folded into the weight as Luna does (BoundedLinearNode.cpp:91-93).
    BoundedLinearNode(const torch::nn::Linear& linear, float alpha = 1.0f, const std::string& name = "");
};

class BoundedConvNode : public BoundedNode {
public:
    BoundedConvNode(const torch::nn::Conv2d& conv, NLR::ConvMode mode = NLR::ConvMode::MATRIX,
                    const std::string& name = "");
};

class BoundedConvTransposeNode : public BoundedNode {
public:
    BoundedConvTransposeNode(const torch::nn::ConvTranspose2d& conv, NLR::ConvMode mode = NLR::ConvMode::MATRIX,
                             const std::string& name = "");
};

class BoundedBatchNormNode : public BoundedNode {
public:
    BoundedBatchNormNode(const torch::Tensor& scale, const torch::Tensor& B, const torch::Tensor& mean,
                         const torch::Tensor& var, float eps, const std::string& name = "");
};

class BoundedReLUNode : public BoundedNode {
public:
    explicit BoundedReLUNode(const torch::nn::ReLU& relu = torch::nn::ReLU(), const std::string& name = "");
};

class BoundedSigmoidNode : public BoundedNode {
public:
    explicit BoundedSigmoidNode(const torch::nn::Sigmoid& s = torch::nn::Sigmoid(), const std::string& name = "");
};

class BoundedAddNode : public BoundedNode {
public:
    BoundedAddNode();
};

class BoundedFlattenNode : public BoundedNode {
public:
    BoundedFlattenNode();
};

class BoundedIdentityNode : public BoundedNode {
public:
    BoundedIdentityNode();
};

// Luna's Reshape flattens (OnnxToTorch.cpp:1959); the engine takes it as a Flatten.
class BoundedReshapeNode : public BoundedNode {
public:
    BoundedReshapeNode();
};

class BoundedSubNode : public BoundedNode {
public:
    BoundedSubNode();
    // BoundedSubNode::setConstantValue (BoundedSubNode.h:54-57).
    void setConstantValue(const torch::Tensor& constant, bool isSecondOperand = true);
};

class BoundedSliceNode : public BoundedNode {
public:
    BoundedSliceNode(int64_t start, int64_t end, int64_t axes, int64_t steps = 1, const std::string& name = "");
};

class BoundedConcatNode : public BoundedNode {
public:
    BoundedConcatNode(int axis, unsigned numInputs, const std::string& name = "");
};

// The engine model behind NLR::TorchModel's interface.
class TorchModel {
public:
    TorchModel(const std::vector<std::shared_ptr<BoundedNode>>& nodes, const std::vector<unsigned>& inputIndices,
               unsigned outputIndex, const std::map<unsigned, std::vector<unsigned>>& dependencies, int device = 0);
    ~TorchModel();
    TorchModel(const TorchModel&) = delete;
    TorchModel& operator=(const TorchModel&) = delete;

    void setInputBounds(const BoundedTensor<torch::Tensor>& inputBounds);
    // C as Luna takes it: [nspec, 1, n_out] (or [nspec, n_out]).
    void setSpecificationMatrix(const torch::Tensor& specMatrix);
    BoundedTensor<torch::Tensor> compute_bounds(const BoundedTensor<torch::Tensor>& input_bounds,
                                                const torch::Tensor* specification_matrix,
                                                LunaConfiguration::AnalysisMethod method, bool bound_lower = true,
                                                bool bound_upper = true);
    BoundedTensor<torch::Tensor> runCROWN(const BoundedTensor<torch::Tensor>& inputBounds);
    BoundedTensor<torch::Tensor> runAlphaCROWN(const BoundedTensor<torch::Tensor>& inputBounds, bool optimizeLower,
                                               bool optimizeUpper);
    BoundedTensor<torch::Tensor> getFinalAnalysisBounds() const { return final_; }
    unsigned getInputSize() const { return n_in_; }
    unsigned getOutputSize() const { return n_out_; }
    // The engine's graph description and its host-only plan (levels, starts,
    // concretisation forms as JSON, lb200_describe_plan).  A model made with
    // device < 0 has only these: no GPU is touched.
    const lb200_graph_desc& graph() const { return graph_; }
    std::string describe() const;

private:
    BoundedTensor<torch::Tensor> run(const BoundedTensor<torch::Tensor>& in, int method, bool lower, bool upper,
                                     bool opt_lower, bool opt_upper);
    std::vector<std::shared_ptr<BoundedNode>> nodes_;
    std::vector<lb200_node_desc> descs_;
    lb200_graph_desc graph_{};
    lb200_model* model_ = nullptr;
    unsigned n_in_ = 0, n_out_ = 0;
    torch::Tensor C_;
    BoundedTensor<torch::Tensor> input_, final_;
};

}  // namespace lb200_luna
