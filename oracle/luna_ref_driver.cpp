// luna_ref_driver.cpp -- test infrastructure, not product code.
//
// A C-ABI driver around Luna's own CPU implementation, compiled from the
// reference sources by oracle/Makefile into oracle/_ref/libluna_ref.so.  It
// is the ground truth that the CPU restatement in oracle/lirpa_oracle.py and
// the CUDA engine are checked against, and the CPU baseline that bench.py
// times.  Nothing in the product links it.
//
// Protocol (fresh state per box, as a Luna user bounding independent boxes
// would do): for every box a new TorchModel is built through the node API,
// mirroring what OnnxToTorchParser builds for Gemm/Relu/Flatten
// (src/input_parsers/OnnxToTorch.cpp:1672-1696,1995,2423), then
// TorchModel::compute_bounds (src/engine/TorchModel.cpp:653-698) is called
// with flat [n] input bounds and C of shape [1, nspec, n_out].
#include "../include/luna_b200.h"

#include "TorchModel.h"
#include "CROWNAnalysis.h"
#include "configuration/LunaConfiguration.h"
#include "nodes/BoundedInputNode.h"
#include "nodes/BoundedLinearNode.h"
#include "nodes/BoundedReLUNode.h"
#include "nodes/BoundedFlattenNode.h"
#include "nodes/BoundedIdentityNode.h"
#include "nodes/BoundedConvNode.h"
#include "nodes/BoundedBatchNormNode.h"
#include "nodes/BoundedConvTransposeNode.h"
#include "nodes/BoundedAddNode.h"
#include "nodes/BoundedSigmoidNode.h"
#include "nodes/BoundedSubNode.h"
#include "nodes/BoundedReshapeNode.h"
#include "nodes/BoundedSliceNode.h"
#include "nodes/BoundedConcatNode.h"
#include "input_parsers/Operations.h"
#include "input_parsers/OutputConstraint.h"
#include "input_parsers/VnnLibInputParser.h"

#include <torch/torch.h>

#include <cstring>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

namespace {

void set_error(char* err, size_t len, const std::string& msg) {
    if (!err || len == 0) return;
    std::strncpy(err, msg.c_str(), len - 1);
    err[len - 1] = '\0';
}

torch::Tensor from_host(const float* p, std::vector<int64_t> shape) {
    auto t = torch::from_blob(const_cast<float*>(p), shape, torch::kFloat32);
    return t.clone();
}

void apply_options(const lb200_options* o) {
    LunaConfiguration::ALPHA_ITERATIONS = o->alpha_iterations;
    LunaConfiguration::ALPHA_LR = o->alpha_lr;
    LunaConfiguration::ALPHA_LR_DECAY = o->alpha_lr_decay;
    LunaConfiguration::EARLY_STOP_PATIENCE = o->early_stop_patience;
    LunaConfiguration::START_SAVE_BEST = o->start_save_best;
    LunaConfiguration::STABILIZE_INTERMEDIATE_BOUNDS = o->stabilize_intermediate_bounds != 0;
    LunaConfiguration::RECOMPUTE_INTERMEDIATE_BOUNDS = o->recompute_intermediate_bounds != 0;
    LunaConfiguration::OPTIMIZE_LOWER = o->optimize_lower != 0;
    LunaConfiguration::OPTIMIZE_UPPER = o->optimize_upper != 0;
    LunaConfiguration::STOP_CROWN_ON_VERIFIED = o->stop_crown_on_verified != 0;
    LunaConfiguration::STOP_ALPHA_ON_VERIFIED = o->stop_alpha_on_verified != 0;
    LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = o->enable_first_linear_ibp != 0;
    LunaConfiguration::USE_STANDARD_CROWN = true;
    LunaConfiguration::USE_PATCHES_MODE = o->use_patches_mode != 0;
    LunaConfiguration::USE_CUDA = false;
    LunaConfiguration::DEVICE = torch::Device(torch::kCPU);
}

std::shared_ptr<NLR::TorchModel> build_model(const lb200_graph_desc* g) {
    Vector<std::shared_ptr<NLR::BoundedTorchNode>> nodes;
    Map<unsigned, Vector<unsigned>> deps;
    for (int i = 0; i < g->num_nodes; ++i) {
        const lb200_node_desc& d = g->nodes[i];
        std::shared_ptr<NLR::BoundedTorchNode> node;
        const int64_t out_numel = (int64_t)d.out_shape[0] * d.out_shape[1] * d.out_shape[2];
        switch (d.type) {
        case LB200_NODE_INPUT:
            node = std::make_shared<NLR::BoundedInputNode>(0, (unsigned)out_numel, "input");
            break;
        case LB200_NODE_LINEAR: {
            torch::nn::Linear lin(torch::nn::LinearOptions(d.in_features, d.out_features));
            lin->weight = from_host(d.weight, {d.out_features, d.in_features});
            lin->bias = d.bias ? from_host(d.bias, {d.out_features})
                               : torch::zeros({d.out_features});
            node = std::make_shared<NLR::BoundedLinearNode>(lin, d.scale, String("linear"));
            node->setInputSize((unsigned)d.in_features);
            node->setOutputSize((unsigned)d.out_features);
            break;
        }
        case LB200_NODE_CONV: {
            // OnnxToTorchParser's Conv2d branch (OnnxToTorch.cpp:2425-2444 and
            // the size/shape setters after it, :2446-2540): MATRIX mode, flat
            // sizes and [1, C, H, W] shapes.
            const lb200_node_desc& src = g->nodes[d.inputs[0]];
            const int64_t Ci = src.out_shape[0], H = src.out_shape[1], W = src.out_shape[2];
            const int64_t Co = d.out_shape[0], kh = d.kernel[0], kw = d.kernel[1];
            torch::nn::Conv2dOptions co(Ci, Co, {kh, kw});
            co.stride({(int64_t)d.stride[0], (int64_t)d.stride[1]});
            co.padding(torch::ExpandingArray<2>({(int64_t)d.padding[0], (int64_t)d.padding[1]}));
            co.bias(d.bias != nullptr);
            torch::nn::Conv2d conv(co);
            conv->weight = from_host(d.weight, {Co, Ci, kh, kw});
            if (d.bias) conv->bias = from_host(d.bias, {Co});
            auto cn = std::make_shared<NLR::BoundedConvNode>(conv, NLR::ConvMode::MATRIX);
            cn->setInputSize((unsigned)(Ci * H * W));
            cn->setOutputSize((unsigned)out_numel);
            cn->setInputShape({1, (int)Ci, (int)H, (int)W});
            cn->setOutputShape({1, (int)Co, d.out_shape[1], d.out_shape[2]});
            node = cn;
            break;
        }
        case LB200_NODE_CONVTRANSPOSE: {
            // OnnxToTorchParser's ConvTranspose (OnnxToTorch.cpp:2680-2717): weight
            // [Ci, Co, kh, kw], MATRIX mode.
            const lb200_node_desc& src = g->nodes[d.inputs[0]];
            const int64_t Ci = src.out_shape[0];
            const int64_t Co = d.out_shape[0], kh = d.kernel[0], kw = d.kernel[1];
            torch::nn::ConvTranspose2dOptions co(Ci, Co, {kh, kw});
            co.stride({(int64_t)d.stride[0], (int64_t)d.stride[1]});
            co.padding(torch::ExpandingArray<2>({(int64_t)d.padding[0], (int64_t)d.padding[1]}));
            co.output_padding(torch::ExpandingArray<2>({(int64_t)d.output_padding[0], (int64_t)d.output_padding[1]}));
            co.bias(d.bias != nullptr);
            torch::nn::ConvTranspose2d ct(co);
            ct->weight = from_host(d.weight, {Ci, Co, kh, kw});
            if (d.bias) ct->bias = from_host(d.bias, {Co});
            auto tn = std::make_shared<NLR::BoundedConvTransposeNode>(ct, NLR::ConvMode::MATRIX);
            // Sizes as a forward pass would leave them (a start at this node
            // sizes its one-hot rows with getOutputSize()).
            tn->setInputSize((unsigned)(Ci * src.out_shape[1] * src.out_shape[2]));
            tn->setOutputSize((unsigned)out_numel);
            node = tn;
            break;
        }
        case LB200_NODE_BATCHNORM: {
            // OnnxToTorchParser's BatchNormalization (OnnxToTorch.cpp:2173-2200):
            // per-channel scale, B, mean, var; flat sizes.
            const int64_t C = d.out_shape[0];
            auto bn = std::make_shared<NLR::BoundedBatchNormNode>(
                from_host(d.weight, {C}), from_host(d.bias, {C}), from_host(d.running_mean, {C}),
                from_host(d.running_var, {C}), d.eps);
            bn->setInputSize((unsigned)out_numel);
            bn->setOutputSize((unsigned)out_numel);
            node = bn;
            break;
        }
        case LB200_NODE_RELU:
            node = std::make_shared<NLR::BoundedReLUNode>(torch::nn::ReLU(), String("relu"));
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        case LB200_NODE_SIGMOID:
            // BoundedOperationConverter::convertSigmoid (OnnxToTorch.cpp:2013-2035).
            node = std::make_shared<NLR::BoundedSigmoidNode>(torch::nn::Sigmoid());
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        case LB200_NODE_FLATTEN:
            node = std::make_shared<NLR::BoundedFlattenNode>(Operations::FlattenWrapper(1));
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        case LB200_NODE_ADD:
            // BoundedOperationConverter::convertAdd for two tensors (OnnxToTorch.cpp:1769-1830):
            // a BoundedAddNode with both producers as dependencies, flat sizes.
            node = std::make_shared<NLR::BoundedAddNode>();
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        case LB200_NODE_IDENTITY:
            node = std::make_shared<NLR::BoundedIdentityNode>(torch::nn::Identity());
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        case LB200_NODE_SUB: {
            // BoundedOperationConverter::convertSub with one constant operand
            // (OnnxToTorch.cpp:2064-2100): setConstantValue(c, constant second?).
            const lb200_node_desc& src = g->nodes[d.inputs[0]];
            const int64_t n_src = (int64_t)src.out_shape[0] * src.out_shape[1] * src.out_shape[2];
            auto sn = std::make_shared<NLR::BoundedSubNode>();
            sn->setConstantValue(from_host(d.constant, {n_src}), d.constant_second != 0);
            sn->setInputSize((unsigned)n_src);
            sn->setOutputSize((unsigned)out_numel);
            node = sn;
            break;
        }
        case LB200_NODE_RESHAPE: {
            // convertReshape (OnnxToTorch.cpp:1935-1972): shape -1, sizes set.
            node = std::make_shared<NLR::BoundedReshapeNode>(Operations::ReshapeWrapper(torch::tensor({-1})));
            node->setInputSize((unsigned)out_numel);
            node->setOutputSize((unsigned)out_numel);
            break;
        }
        case LB200_NODE_SLICE: {
            // convertSlice (OnnxToTorch.cpp:2924): BoundedSliceNode(start, end, axes, steps).
            const lb200_node_desc& src = g->nodes[d.inputs[0]];
            node = std::make_shared<NLR::BoundedSliceNode>(d.start, d.end, (int64_t)d.axis, d.step, String("slice"));
            node->setInputSize((unsigned)((int64_t)src.out_shape[0] * src.out_shape[1] * src.out_shape[2]));
            node->setOutputSize((unsigned)out_numel);
            break;
        }
        case LB200_NODE_CONCAT: {
            // convertConcat (OnnxToTorch.cpp:2734): BoundedConcatNode(axis, numInputs).
            auto cn = std::make_shared<NLR::BoundedConcatNode>((int)d.axis, (unsigned)d.num_inputs);
            cn->setInputSize((unsigned)out_numel);
            cn->setOutputSize((unsigned)out_numel);
            node = cn;
            break;
        }
        default:
            throw std::runtime_error("luna_ref_driver: node type " + std::to_string(d.type) +
                                     " is not wired into the reference driver");
        }
        node->setNodeIndex((unsigned)i);
        nodes.append(node);
        Vector<unsigned> dv;
        for (int k = 0; k < d.num_inputs; ++k) dv.append((unsigned)d.inputs[k]);
        deps[(unsigned)i] = dv;
    }
    Vector<unsigned> inputs;
    inputs.append((unsigned)g->input_index);
    return std::make_shared<NLR::TorchModel>(nodes, inputs, (unsigned)g->output_index, deps);
}

bool feeds_relu(const lb200_graph_desc* g, int node) {
    for (int i = 0; i < g->num_nodes; ++i) {
        const lb200_node_desc& d = g->nodes[i];
        if (d.type != LB200_NODE_RELU && d.type != LB200_NODE_SIGMOID) continue;
        if (d.num_inputs > 0 && d.inputs[0] == node) return true;
    }
    return false;
}

}  // namespace

extern "C" {

// Number of floats per box in the intermediate-bound dump: every node that
// feeds an activation, in node-id order.
int64_t luna_ref_intermediate_size(const lb200_graph_desc* g) {
    int64_t n = 0;
    for (int i = 0; i < g->num_nodes; ++i)
        if (feeds_relu(g, i))
            n += (int64_t)g->nodes[i].out_shape[0] * g->nodes[i].out_shape[1] * g->nodes[i].out_shape[2];
    return n;
}

// Bound boxes [box_begin, box_end) with Luna.  inter_lb / inter_ub may be
// NULL; otherwise they receive [n_boxes, luna_ref_intermediate_size] floats.
int luna_ref_compute_bounds(const lb200_graph_desc* g, const lb200_options* opt, int method,
                            const float* x_lower, const float* x_upper, int64_t n_boxes,
                            int64_t n_in, const float* C, int64_t c_boxes, int64_t nspec,
                            int64_t n_out, float* out_lb, float* out_ub, float* inter_lb,
                            float* inter_ub, int num_threads, char* err, size_t errlen) {
    try {
        at::set_num_threads(num_threads > 0 ? num_threads : 1);
        apply_options(opt);
        const int64_t inter_n = luna_ref_intermediate_size(g);
        for (int64_t b = 0; b < n_boxes; ++b) {
            auto model = build_model(g);
            torch::Tensor lb = from_host(x_lower + b * n_in, {n_in});
            torch::Tensor ub = from_host(x_upper + b * n_in, {n_in});
            const float* cb = C + (c_boxes == 1 ? 0 : b) * nspec * n_out;
            torch::Tensor Cm = from_host(cb, {1, nspec, n_out});
            BoundedTensor<torch::Tensor> box(lb, ub);
            torch::Tensor rl, ru;
            if (method == LB200_METHOD_IBP) {
                model->setInputBounds(box);
                NLR::CROWNAnalysis an(model.get());
                an.setInputBounds(box);
                an.computeIBPBounds();
                auto ob = an.getOutputIBPBounds();
                torch::Tensor C2 = Cm.squeeze(0);
                torch::Tensor Cp = torch::clamp_min(C2, 0), Cn = torch::clamp_max(C2, 0);
                rl = Cp.matmul(ob.lower().flatten()) + Cn.matmul(ob.upper().flatten());
                ru = Cp.matmul(ob.upper().flatten()) + Cn.matmul(ob.lower().flatten());
            } else {
                auto m = method == LB200_METHOD_ALPHA_CROWN
                             ? LunaConfiguration::AnalysisMethod::AlphaCROWN
                             : LunaConfiguration::AnalysisMethod::CROWN;
                // compute_bounds mutates these two globals; reset them per box.
                LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
                auto res = model->compute_bounds(box, &Cm, m, true, true);
                rl = res.lower().flatten();
                ru = res.upper().flatten();
            }
            if (rl.numel() != nspec || ru.numel() != nspec)
                throw std::runtime_error("luna_ref_driver: unexpected bound shape");
            std::memcpy(out_lb + b * nspec, rl.contiguous().data_ptr<float>(), nspec * sizeof(float));
            std::memcpy(out_ub + b * nspec, ru.contiguous().data_ptr<float>(), nspec * sizeof(float));
            if (inter_lb && inter_ub && method != LB200_METHOD_IBP) {
                auto state = model->getState();
                int64_t off = 0;
                for (int i = 0; i < g->num_nodes; ++i) {
                    if (!feeds_relu(g, i)) continue;
                    const int64_t sz = (int64_t)g->nodes[i].out_shape[0] * g->nodes[i].out_shape[1] *
                                       g->nodes[i].out_shape[2];
                    auto it = state.allBounds.find((unsigned)i);
                    float* dl = inter_lb + b * inter_n + off;
                    float* du = inter_ub + b * inter_n + off;
                    if (it != state.allBounds.end()) {
                        auto l = it->second.first.flatten().contiguous();
                        auto u = it->second.second.flatten().contiguous();
                        std::memcpy(dl, l.data_ptr<float>(), sz * sizeof(float));
                        std::memcpy(du, u.data_ptr<float>(), sz * sizeof(float));
                    } else {
                        for (int64_t k = 0; k < sz; ++k) { dl[k] = NAN; du[k] = NAN; }
                    }
                    off += sz;
                }
            }
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    } catch (...) {
        set_error(err, errlen, "luna_ref_driver: unknown exception");
        return 1;
    }
}

// ---- Warm start: a child box bounded from its parent's state -------------
//
// As branch-and-bound hands a sub-domain its parent's state: the parent box
// is bounded with alpha-CROWN (TorchModel::compute_bounds), its state taken
// (TorchModel::getState, src/engine/TorchModel.h:123-135) and loaded into the
// same model with the child's input box (TorchModel::loadState), then the
// child is bounded with alpha-CROWN.  parents / children are [n_children,
// n_in] each (child i's parent is parent box i).
int luna_ref_compute_bounds_warm(const lb200_graph_desc* g, const lb200_options* opt, const float* p_lower,
                                 const float* p_upper, const float* c_lower, const float* c_upper,
                                 int64_t n_children, int64_t n_in, const float* C, int64_t c_boxes,
                                 int64_t nspec, int64_t n_out, float* out_lb, float* out_ub, int num_threads,
                                 char* err, size_t errlen) {
    try {
        at::set_num_threads(num_threads > 0 ? num_threads : 1);
        apply_options(opt);
        const auto alpha = LunaConfiguration::AnalysisMethod::AlphaCROWN;
        for (int64_t b = 0; b < n_children; ++b) {
            auto model = build_model(g);
            const float* cb = C + (c_boxes == 1 ? 0 : b) * nspec * n_out;
            torch::Tensor Cm = from_host(cb, {1, nspec, n_out});
            BoundedTensor<torch::Tensor> parent(from_host(p_lower + b * n_in, {n_in}),
                                                from_host(p_upper + b * n_in, {n_in}));
            LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
            model->compute_bounds(parent, &Cm, alpha, true, true);
            auto state = model->getState();
            BoundedTensor<torch::Tensor> child(from_host(c_lower + b * n_in, {n_in}),
                                               from_host(c_upper + b * n_in, {n_in}));
            model->loadState(child, state.allBounds, state.alphas);
            LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
            auto res = model->compute_bounds(child, &Cm, alpha, true, true);
            torch::Tensor rl = res.lower().flatten(), ru = res.upper().flatten();
            if (rl.numel() != nspec || ru.numel() != nspec)
                throw std::runtime_error("luna_ref_driver: unexpected bound shape");
            std::memcpy(out_lb + b * nspec, rl.contiguous().data_ptr<float>(), nspec * sizeof(float));
            std::memcpy(out_ub + b * nspec, ru.contiguous().data_ptr<float>(), nspec * sizeof(float));
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    } catch (...) {
        set_error(err, errlen, "luna_ref_driver: unknown exception");
        return 1;
    }
}

// A chain of warm starts down one path of a split tree, as a
// branch-and-bound driver repeats getState / loadState / compute_bounds
// (Luna's own tests/unit/analysis/test_bab_state.cpp, repeatedLoadStateAndRun):
// for each of n_paths paths, boxes [depth, n_in] from the root down; the
// root is bounded fresh, every later box after loading the state the one
// above it left.  out_lb / out_ub receive [n_paths, depth, nspec]; C is
// [1 or n_paths, nspec, n_out] (one specification per path).
int luna_ref_compute_bounds_chain(const lb200_graph_desc* g, const lb200_options* opt, const float* lower,
                                  const float* upper, int64_t n_paths, int64_t depth, int64_t n_in, const float* C,
                                  int64_t c_boxes, int64_t nspec, int64_t n_out, float* out_lb, float* out_ub,
                                  int num_threads, char* err, size_t errlen) {
    try {
        at::set_num_threads(num_threads > 0 ? num_threads : 1);
        apply_options(opt);
        const auto alpha = LunaConfiguration::AnalysisMethod::AlphaCROWN;
        for (int64_t p = 0; p < n_paths; ++p) {
            auto model = build_model(g);
            const float* cb = C + (c_boxes == 1 ? 0 : p) * nspec * n_out;
            torch::Tensor Cm = from_host(cb, {1, nspec, n_out});
            for (int64_t d = 0; d < depth; ++d) {
                const int64_t at_box = (p * depth + d) * n_in;
                BoundedTensor<torch::Tensor> box(from_host(lower + at_box, {n_in}), from_host(upper + at_box, {n_in}));
                if (d > 0) {
                    auto state = model->getState();
                    model->loadState(box, state.allBounds, state.alphas);
                }
                LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
                auto res = model->compute_bounds(box, &Cm, alpha, true, true);
                torch::Tensor rl = res.lower().flatten(), ru = res.upper().flatten();
                if (rl.numel() != nspec || ru.numel() != nspec)
                    throw std::runtime_error("luna_ref_driver: unexpected bound shape");
                std::memcpy(out_lb + (p * depth + d) * nspec, rl.contiguous().data_ptr<float>(), nspec * sizeof(float));
                std::memcpy(out_ub + (p * depth + d) * nspec, ru.contiguous().data_ptr<float>(), nspec * sizeof(float));
            }
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    } catch (...) {
        set_error(err, errlen, "luna_ref_driver: unknown exception");
        return 1;
    }
}

// ---- VNN-LIB properties through Luna's own parser ------------------------
//
// As TorchModel(onnxPath, vnnlibPath) reads a property
// (src/engine/TorchModelOnnxFactory.cpp:89-192): parseInputBounds (a failure
// fails the call, return 2), then parseOutputConstraints + toCMatrix when
// there are constraints (a failure drops the specification:
// *spec_dropped = 1).  C [cap_rows, n_out], thresholds and branch [cap_rows]
// receive up to cap_rows rows; *nspec is the true count (return 3 when it
// exceeds cap_rows).  *n_branches is 0 without OR branches.
int luna_ref_vnnlib_parse(const char* path, int64_t n_in, int64_t n_out, float* lower, float* upper,
                          int64_t cap_rows, float* C, float* thresholds, int32_t* branch, int64_t* nspec,
                          int32_t* n_branches, int32_t* spec_dropped, char* err, size_t errlen) {
    *nspec = 0;
    *n_branches = 0;
    *spec_dropped = 0;
    try {
        auto ib = VnnLibInputParser::parseInputBounds(String(path), (unsigned)n_in);
        auto lo = ib.lower().contiguous(), hi = ib.upper().contiguous();
        std::memcpy(lower, lo.data_ptr<float>(), n_in * sizeof(float));
        std::memcpy(upper, hi.data_ptr<float>(), n_in * sizeof(float));
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 2;
    }
    try {
        auto oc = VnnLibInputParser::parseOutputConstraints(String(path), (unsigned)n_out);
        if (!oc.hasConstraints()) return 0;
        auto r = oc.toCMatrix();
        const int64_t rows = r.C.size(0);
        *nspec = rows;
        *n_branches = r.hasORBranches ? (int32_t)r.branchSizes.size() : 0;
        if (rows > cap_rows) return 3;
        auto c = r.C.reshape({rows, n_out}).contiguous();
        auto t = r.thresholds.contiguous();
        std::memcpy(C, c.data_ptr<float>(), rows * n_out * sizeof(float));
        std::memcpy(thresholds, t.data_ptr<float>(), rows * sizeof(float));
        for (int64_t k = 0; k < rows; ++k) branch[k] = r.hasORBranches ? (int32_t)r.branchMapping[(unsigned)k] : 0;
        return 0;
    } catch (const std::exception& e) {
        *nspec = 0;
        *n_branches = 0;
        *spec_dropped = 1;
        set_error(err, errlen, e.what());
        return 0;
    }
}

}  // extern "C"

namespace {

// The CLI's verdict (src/engine/LunaMain.cpp:60-135, a static function of
// the CLI, restated here): OR branches through Luna's own
// OutputConstraintSet::evaluateORBranches, a conjunction by its two tests.
int ref_status(const torch::Tensor& lb, const torch::Tensor& ub, const torch::Tensor& thr,
               const Vector<unsigned>& mapping, const Vector<unsigned>& sizes, bool has_or) {
    if (lb.numel() == 0 || ub.numel() == 0) return LB200_STATUS_UNKNOWN;
    if (lb.numel() != thr.numel() || ub.numel() != thr.numel()) return LB200_STATUS_UNKNOWN;
    if (has_or) {
        auto res = NLR::OutputConstraintSet::evaluateORBranches(lb, ub, thr, mapping, sizes);
        bool all_disproved = true, any_sat = false;
        for (const auto& b : res) {
            if (!b.verified) all_disproved = false;
            if (b.refuted) any_sat = true;
        }
        if (all_disproved) return LB200_STATUS_UNSAT;
        return any_sat ? LB200_STATUS_SAT : LB200_STATUS_UNKNOWN;
    }
    if ((lb - thr > 0).any().item<bool>()) return LB200_STATUS_UNSAT;
    if ((ub - thr <= 0).all().item<bool>()) return LB200_STATUS_SAT;
    return LB200_STATUS_UNKNOWN;
}

torch::Tensor rows_tensor(const float* p, int64_t n) { return from_host(p, {n}); }

}  // namespace

extern "C" {

// Luna's verdict for n_boxes boxes of bounds [n_boxes, nspec]
// (n_branches == 0: a conjunction).
int luna_ref_property_status(const float* lb, const float* ub, int64_t n_boxes, int64_t nspec,
                             const float* thresholds, const int32_t* branch, int32_t n_branches, int32_t* status,
                             char* err, size_t errlen) {
    try {
        Vector<unsigned> mapping, sizes;
        for (int64_t k = 0; k < nspec && n_branches > 0; ++k) mapping.append((unsigned)branch[k]);
        for (int32_t b = 0; b < n_branches; ++b) {
            unsigned cnt = 0;
            for (int64_t k = 0; k < nspec; ++k) cnt += branch[k] == b;
            sizes.append(cnt);
        }
        torch::Tensor thr = rows_tensor(thresholds, nspec);
        for (int64_t b = 0; b < n_boxes; ++b)
            status[b] = ref_status(rows_tensor(lb + b * nspec, nspec), rows_tensor(ub + b * nspec, nspec), thr,
                                   mapping, sizes, n_branches > 0);
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    }
}

// The CLI's flow for each box (src/engine/LunaMain.cpp:240-330): a fresh
// model, the property's constraints set with setSpecificationFromConstraints
// (thresholds and branches kept, so STOP_*_ON_VERIFIED apply), then
// compute_bounds(box, nullptr, method, true, true) and the verdict.  The
// constraints arrive as the rows Luna's toCMatrix made of them (C
// [nspec, n_out], thresholds, branch of each row, n_branches == 0 for a
// conjunction) and are rebuilt into an OutputConstraintSet: Luna's
// tokenizer (std::regex) cannot run inside a Python process that has
// imported torch, so the text is parsed out of process.  nspec == 0: no
// specification, out_lb / out_ub are [n_boxes, n_out] and status UNKNOWN.
int luna_ref_compute_property(const lb200_graph_desc* g, const lb200_options* opt, int method, const float* C,
                              const float* thresholds, const int32_t* branch, int64_t nspec, int32_t n_branches,
                              const float* x_lower, const float* x_upper, int64_t n_boxes, int64_t n_in,
                              int64_t n_out, float* out_lb, float* out_ub, int32_t* status, int num_threads,
                              char* err, size_t errlen) {
    try {
        at::set_num_threads(num_threads > 0 ? num_threads : 1);
        apply_options(opt);
        NLR::OutputConstraintSet oc;
        oc.setOutputDimension((unsigned)n_out);
        auto row = [&](int64_t r) {
            NLR::OutputConstraint c;
            for (int64_t j = 0; j < n_out; ++j)
                if (C[r * n_out + j] != 0.f) c.terms.append(NLR::OutputTerm((unsigned)j, C[r * n_out + j]));
            c.threshold = thresholds[r];
            return c;
        };
        if (n_branches > 0) {
            for (int32_t b = 0; b < n_branches; ++b) {
                Vector<NLR::OutputConstraint> br;
                for (int64_t r = 0; r < nspec; ++r)
                    if (branch[r] == b) br.append(row(r));
                oc.addORBranch(br);
            }
        } else {
            for (int64_t r = 0; r < nspec; ++r) oc.addConstraint(row(r));
        }
        const bool spec = nspec > 0;
        NLR::CMatrixResult cm;
        if (spec) cm = oc.toCMatrix();
        // The reference reports early stops on std::cout with numbers in
        // them; number formatting through std::cout crashes when the library
        // is loaded into a Python process, so the stream is muted (a stream
        // in a failed state formats nothing) for the duration of the call.
        struct Mute {
            std::ios_base::iostate was = std::cout.rdstate();
            Mute() { std::cout.setstate(std::ios_base::badbit); }
            ~Mute() { std::cout.clear(was); }
        } mute;
        for (int64_t b = 0; b < n_boxes; ++b) {
            auto model = build_model(g);
            if (spec) model->setSpecificationFromConstraints(oc);
            BoundedTensor<torch::Tensor> box(from_host(x_lower + b * n_in, {n_in}),
                                             from_host(x_upper + b * n_in, {n_in}));
            LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
            auto m = method == LB200_METHOD_ALPHA_CROWN ? LunaConfiguration::AnalysisMethod::AlphaCROWN
                                                         : LunaConfiguration::AnalysisMethod::CROWN;
            auto res = model->compute_bounds(box, nullptr, m, true, true);
            torch::Tensor rl = res.lower().flatten().contiguous(), ru = res.upper().flatten().contiguous();
            const int64_t rows = spec ? nspec : n_out;
            if (rl.numel() != rows || ru.numel() != rows)
                throw std::runtime_error("luna_ref_driver: unexpected bound shape");
            std::memcpy(out_lb + b * rows, rl.data_ptr<float>(), rows * sizeof(float));
            std::memcpy(out_ub + b * rows, ru.data_ptr<float>(), rows * sizeof(float));
            status[b] = spec ? ref_status(rl, ru, cm.thresholds, cm.branchMapping, cm.branchSizes, cm.hasORBranches)
                             : LB200_STATUS_UNKNOWN;
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    } catch (...) {
        set_error(err, errlen, "luna_ref_driver: unknown exception");
        return 1;
    }
}

}  // extern "C"
