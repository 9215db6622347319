// luna_shim_check.cpp -- test infrastructure, not product code.
//
// Checks the Luna-side shim (luna_b200_shim.h) the way a Luna front end
// would use it: for one graph description, torch modules are made and
// handed both to Luna's own node constructors (an NLR::TorchModel, Luna's
// CPU path) and to the shim's (an lb200_luna::TorchModel, the B200 engine),
// exactly as OnnxToTorchParser would build the two side by side
// (OnnxToTorch.cpp:1672-1696,2173-2200,2425-2444,2680-2717).  Both models
// bound the same box through TorchModel::compute_bounds; the caller compares
// the results.  Luna's CPU path picks the patches form for every conv start
// when CUDA is available to its process (CROWNAnalysis.cpp:261-271) and by a
// 4096-feature threshold otherwise, so a caller on a GPU host runs Luna's
// side (`which` = 1) in a process with CUDA hidden and the shim's (`which` =
// 2) in its own.  Built by oracle/Makefile into oracle/_ref/libluna_shim_check.so.
#include "luna_b200_shim.h"

#include "TorchModel.h"
#include "input_parsers/Operations.h"
#include "nodes/BoundedAddNode.h"
#include "nodes/BoundedBatchNormNode.h"
#include "nodes/BoundedConvNode.h"
#include "nodes/BoundedConvTransposeNode.h"
#include "nodes/BoundedFlattenNode.h"
#include "nodes/BoundedIdentityNode.h"
#include "nodes/BoundedInputNode.h"
#include "nodes/BoundedLinearNode.h"
#include "nodes/BoundedReLUNode.h"
#include "nodes/BoundedSigmoidNode.h"
#include "nodes/BoundedConcatNode.h"
#include "nodes/BoundedReshapeNode.h"
#include "nodes/BoundedSliceNode.h"
#include "nodes/BoundedSubNode.h"

#include <cstring>

namespace {

torch::Tensor from_host(const float* p, std::vector<int64_t> shape) {
    return torch::from_blob(const_cast<float*>(p), shape, torch::kFloat32).clone();
}

struct Both {
    std::shared_ptr<NLR::BoundedTorchNode> luna;
    std::shared_ptr<lb200_luna::BoundedNode> shim;
};

Both make_node(const lb200_graph_desc* g, int i) {
    const lb200_node_desc& d = g->nodes[i];
    const int64_t numel = (int64_t)d.out_shape[0] * d.out_shape[1] * d.out_shape[2];
    Both b;
    switch (d.type) {
    case LB200_NODE_INPUT: {
        b.luna = std::make_shared<NLR::BoundedInputNode>(0, (unsigned)numel, "input");
        auto s = std::make_shared<lb200_luna::BoundedInputNode>(0, (unsigned)numel, "input");
        s->setOutputShape({1, d.out_shape[0], d.out_shape[1], d.out_shape[2]});
        b.shim = s;
        break;
    }
    case LB200_NODE_LINEAR: {
        torch::nn::Linear lin(torch::nn::LinearOptions(d.in_features, d.out_features));
        lin->weight = from_host(d.weight, {d.out_features, d.in_features});
        lin->bias = d.bias ? from_host(d.bias, {d.out_features}) : torch::zeros({d.out_features});
        b.luna = std::make_shared<NLR::BoundedLinearNode>(lin, d.scale, String("linear"));
        b.luna->setInputSize((unsigned)d.in_features);
        b.luna->setOutputSize((unsigned)d.out_features);
        b.shim = std::make_shared<lb200_luna::BoundedLinearNode>(lin, d.scale, "linear");
        break;
    }
    case LB200_NODE_CONV: {
        const lb200_node_desc& src = g->nodes[d.inputs[0]];
        const int64_t Ci = src.out_shape[0], H = src.out_shape[1], W = src.out_shape[2];
        const int64_t Co = d.out_shape[0];
        torch::nn::Conv2dOptions co(Ci, Co, {(int64_t)d.kernel[0], (int64_t)d.kernel[1]});
        co.stride({(int64_t)d.stride[0], (int64_t)d.stride[1]});
        co.padding(torch::ExpandingArray<2>({(int64_t)d.padding[0], (int64_t)d.padding[1]}));
        co.bias(d.bias != nullptr);
        torch::nn::Conv2d conv(co);
        conv->weight = from_host(d.weight, {Co, Ci, (int64_t)d.kernel[0], (int64_t)d.kernel[1]});
        if (d.bias) conv->bias = from_host(d.bias, {Co});
        auto cn = std::make_shared<NLR::BoundedConvNode>(conv, NLR::ConvMode::MATRIX);
        cn->setInputSize((unsigned)(Ci * H * W));
        cn->setOutputSize((unsigned)numel);
        cn->setInputShape({1, (int)Ci, (int)H, (int)W});
        cn->setOutputShape({1, (int)Co, d.out_shape[1], d.out_shape[2]});
        b.luna = cn;
        auto s = std::make_shared<lb200_luna::BoundedConvNode>(conv, NLR::ConvMode::MATRIX);
        s->setOutputShape({1, (int)Co, d.out_shape[1], d.out_shape[2]});
        b.shim = s;
        break;
    }
    case LB200_NODE_CONVTRANSPOSE: {
        const lb200_node_desc& src = g->nodes[d.inputs[0]];
        const int64_t Ci = src.out_shape[0], Co = d.out_shape[0];
        torch::nn::ConvTranspose2dOptions co(Ci, Co, {(int64_t)d.kernel[0], (int64_t)d.kernel[1]});
        co.stride({(int64_t)d.stride[0], (int64_t)d.stride[1]});
        co.padding(torch::ExpandingArray<2>({(int64_t)d.padding[0], (int64_t)d.padding[1]}));
        co.bias(d.bias != nullptr);
        torch::nn::ConvTranspose2d ct(co);
        ct->weight = from_host(d.weight, {Ci, Co, (int64_t)d.kernel[0], (int64_t)d.kernel[1]});
        if (d.bias) ct->bias = from_host(d.bias, {Co});
        b.luna = std::make_shared<NLR::BoundedConvTransposeNode>(ct, NLR::ConvMode::MATRIX);
        b.luna->setInputSize((unsigned)(Ci * src.out_shape[1] * src.out_shape[2]));
        b.luna->setOutputSize((unsigned)numel);
        auto s = std::make_shared<lb200_luna::BoundedConvTransposeNode>(ct, NLR::ConvMode::MATRIX);
        s->setOutputShape({1, (int)Co, d.out_shape[1], d.out_shape[2]});
        b.shim = s;
        break;
    }
    case LB200_NODE_BATCHNORM: {
        const int64_t C = d.out_shape[0];
        auto scale = from_host(d.weight, {C}), B = from_host(d.bias, {C});
        auto mean = from_host(d.running_mean, {C}), var = from_host(d.running_var, {C});
        b.luna = std::make_shared<NLR::BoundedBatchNormNode>(scale, B, mean, var, d.eps);
        b.luna->setInputSize((unsigned)numel);
        b.luna->setOutputSize((unsigned)numel);
        b.shim = std::make_shared<lb200_luna::BoundedBatchNormNode>(scale, B, mean, var, d.eps);
        break;
    }
    case LB200_NODE_RELU:
        b.luna = std::make_shared<NLR::BoundedReLUNode>(torch::nn::ReLU(), String("relu"));
        b.shim = std::make_shared<lb200_luna::BoundedReLUNode>();
        break;
    case LB200_NODE_SIGMOID:
        b.luna = std::make_shared<NLR::BoundedSigmoidNode>(torch::nn::Sigmoid());
        b.shim = std::make_shared<lb200_luna::BoundedSigmoidNode>();
        break;
    case LB200_NODE_FLATTEN:
        b.luna = std::make_shared<NLR::BoundedFlattenNode>(Operations::FlattenWrapper(1));
        b.shim = std::make_shared<lb200_luna::BoundedFlattenNode>();
        break;
    case LB200_NODE_ADD:
        b.luna = std::make_shared<NLR::BoundedAddNode>();
        b.shim = std::make_shared<lb200_luna::BoundedAddNode>();
        break;
    case LB200_NODE_IDENTITY:
        b.luna = std::make_shared<NLR::BoundedIdentityNode>(torch::nn::Identity());
        b.shim = std::make_shared<lb200_luna::BoundedIdentityNode>();
        break;
    case LB200_NODE_SUB: {
        const lb200_node_desc& src = g->nodes[d.inputs[0]];
        const int64_t n_src = (int64_t)src.out_shape[0] * src.out_shape[1] * src.out_shape[2];
        auto c = from_host(d.constant, {n_src});
        auto ln = std::make_shared<NLR::BoundedSubNode>();
        ln->setConstantValue(c, d.constant_second != 0);
        b.luna = ln;
        auto sn = std::make_shared<lb200_luna::BoundedSubNode>();
        sn->setConstantValue(c, d.constant_second != 0);
        b.shim = sn;
        break;
    }
    case LB200_NODE_RESHAPE:
        b.luna = std::make_shared<NLR::BoundedReshapeNode>(Operations::ReshapeWrapper(torch::tensor({-1})));
        b.shim = std::make_shared<lb200_luna::BoundedReshapeNode>();
        break;
    case LB200_NODE_SLICE: {
        b.luna = std::make_shared<NLR::BoundedSliceNode>(d.start, d.end, (int64_t)d.axis, d.step, String("slice"));
        auto sn = std::make_shared<lb200_luna::BoundedSliceNode>(d.start, d.end, (int64_t)d.axis, d.step);
        sn->setOutputShape({1, d.out_shape[0], d.out_shape[1], d.out_shape[2]});
        b.shim = sn;
        break;
    }
    case LB200_NODE_CONCAT: {
        b.luna = std::make_shared<NLR::BoundedConcatNode>((int)d.axis, (unsigned)d.num_inputs);
        auto sn = std::make_shared<lb200_luna::BoundedConcatNode>((int)d.axis, (unsigned)d.num_inputs);
        sn->setOutputShape({1, d.out_shape[0], d.out_shape[1], d.out_shape[2]});
        b.shim = sn;
        break;
    }
    default:
        throw std::runtime_error("luna_shim_check: node type " + std::to_string(d.type) + " not wired");
    }
    if (d.type == LB200_NODE_RELU || d.type == LB200_NODE_SIGMOID || d.type == LB200_NODE_FLATTEN ||
        d.type == LB200_NODE_ADD || d.type == LB200_NODE_IDENTITY || d.type == LB200_NODE_SUB ||
        d.type == LB200_NODE_RESHAPE || d.type == LB200_NODE_SLICE || d.type == LB200_NODE_CONCAT) {
        b.luna->setInputSize((unsigned)numel);
        b.luna->setOutputSize((unsigned)numel);
    }
    b.luna->setNodeIndex((unsigned)i);
    return b;
}

void set_error(char* err, size_t len, const std::string& msg) {
    if (!err || len == 0) return;
    std::strncpy(err, msg.c_str(), len - 1);
    err[len - 1] = '\0';
}

}  // namespace

extern "C" {

// One box through Luna's model (which & 1) and the shim's (which & 2, on
// CUDA device `device`).  method: LB200_METHOD_CROWN or
// LB200_METHOD_ALPHA_CROWN; C [nspec, n_out]; results [nspec] each.  The
// LunaConfiguration flags are set from `opt` before each model runs.
int luna_shim_check(const lb200_graph_desc* g, const lb200_options* opt, int method, const float* x_lower,
                    const float* x_upper, int64_t n_in, const float* C, int64_t nspec, int64_t n_out, int device,
                    int which, float* luna_lb, float* luna_ub, float* shim_lb, float* shim_ub, char* err,
                    size_t errlen) {
    try {
        at::set_num_threads(1);
        auto configure = [&] {
        LunaConfiguration::ALPHA_ITERATIONS = opt->alpha_iterations;
        LunaConfiguration::ALPHA_LR = opt->alpha_lr;
        LunaConfiguration::ALPHA_LR_DECAY = opt->alpha_lr_decay;
        LunaConfiguration::EARLY_STOP_PATIENCE = opt->early_stop_patience;
        LunaConfiguration::START_SAVE_BEST = opt->start_save_best;
        LunaConfiguration::STABILIZE_INTERMEDIATE_BOUNDS = opt->stabilize_intermediate_bounds != 0;
        LunaConfiguration::RECOMPUTE_INTERMEDIATE_BOUNDS = opt->recompute_intermediate_bounds != 0;
        LunaConfiguration::OPTIMIZE_LOWER = opt->optimize_lower != 0;
        LunaConfiguration::OPTIMIZE_UPPER = opt->optimize_upper != 0;
        LunaConfiguration::STOP_CROWN_ON_VERIFIED = opt->stop_crown_on_verified != 0;
        LunaConfiguration::STOP_ALPHA_ON_VERIFIED = opt->stop_alpha_on_verified != 0;
        LunaConfiguration::ENABLE_FIRST_LINEAR_IBP = opt->enable_first_linear_ibp != 0;
        LunaConfiguration::USE_STANDARD_CROWN = true;
        LunaConfiguration::USE_PATCHES_MODE = opt->use_patches_mode != 0;
        LunaConfiguration::USE_CUDA = false;
        LunaConfiguration::DEVICE = torch::Device(torch::kCPU);
        };

        Vector<std::shared_ptr<NLR::BoundedTorchNode>> luna_nodes;
        Map<unsigned, Vector<unsigned>> luna_deps;
        std::vector<std::shared_ptr<lb200_luna::BoundedNode>> shim_nodes;
        std::map<unsigned, std::vector<unsigned>> shim_deps;
        for (int i = 0; i < g->num_nodes; ++i) {
            Both b = make_node(g, i);
            luna_nodes.append(b.luna);
            shim_nodes.push_back(b.shim);
            Vector<unsigned> dv;
            std::vector<unsigned> sv;
            for (int k = 0; k < g->nodes[i].num_inputs; ++k) {
                dv.append((unsigned)g->nodes[i].inputs[k]);
                sv.push_back((unsigned)g->nodes[i].inputs[k]);
            }
            luna_deps[(unsigned)i] = dv;
            shim_deps[(unsigned)i] = sv;
        }
        Vector<unsigned> luna_in;
        luna_in.append((unsigned)g->input_index);
        const auto am = method == LB200_METHOD_ALPHA_CROWN ? LunaConfiguration::AnalysisMethod::AlphaCROWN
                                                          : LunaConfiguration::AnalysisMethod::CROWN;
        BoundedTensor<torch::Tensor> box(from_host(x_lower, {n_in}), from_host(x_upper, {n_in}));
        torch::Tensor spec = from_host(C, {nspec, 1, n_out});
        auto put = [&](const torch::Tensor& t, float* dst) {
            auto c = t.detach().to(torch::kFloat32).contiguous().reshape({-1});
            if (c.numel() != nspec) throw std::runtime_error("unexpected result size");
            std::memcpy(dst, c.data_ptr<float>(), (size_t)nspec * 4);
        };
        if (which & 1) {
            configure();
            NLR::TorchModel luna(luna_nodes, luna_in, (unsigned)g->output_index, luna_deps);
            auto rl = luna.compute_bounds(box, &spec, am, true, true);
            put(rl.lower(), luna_lb);
            put(rl.upper(), luna_ub);
        }
        if (which & 2) {
            configure();
            lb200_luna::TorchModel shim(shim_nodes, {(unsigned)g->input_index}, (unsigned)g->output_index, shim_deps,
                                        device);
            auto rs = shim.compute_bounds(box, &spec, am, true, true);
            put(rs.lower(), shim_lb);
            put(rs.upper(), shim_ub);
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    }
}

// The shim's graph description of `g` (built as luna_shim_check builds it,
// no GPU): node kinds, producers, shapes and, per node, the sum of its
// weight and bias arrays, for comparison with the description the caller
// made directly.  out: [num_nodes, 12] doubles; raw (may be null): the
// descriptors themselves, [num_nodes] lb200_node_desc.
int luna_shim_describe(const lb200_graph_desc* g, double* out, lb200_node_desc* raw, char* err, size_t errlen) {
    try {
        std::vector<std::shared_ptr<lb200_luna::BoundedNode>> shim_nodes;
        std::map<unsigned, std::vector<unsigned>> shim_deps;
        for (int i = 0; i < g->num_nodes; ++i) {
            shim_nodes.push_back(make_node(g, i).shim);
            std::vector<unsigned> sv;
            for (int k = 0; k < g->nodes[i].num_inputs; ++k) sv.push_back((unsigned)g->nodes[i].inputs[k]);
            shim_deps[(unsigned)i] = sv;
        }
        lb200_luna::TorchModel shim(shim_nodes, {(unsigned)g->input_index}, (unsigned)g->output_index, shim_deps, -1);
        const lb200_graph_desc& d = shim.graph();
        if (raw) std::memcpy(raw, d.nodes, sizeof(lb200_node_desc) * d.num_nodes);
        for (int i = 0; i < d.num_nodes; ++i) {
            const lb200_node_desc& n = d.nodes[i];
            double* o = out + 12 * i;
            o[0] = n.type;
            o[1] = n.num_inputs;
            o[2] = n.num_inputs > 0 ? n.inputs[0] : -1;
            o[3] = n.num_inputs > 1 ? n.inputs[1] : -1;
            o[4] = n.out_shape[0];
            o[5] = n.out_shape[1];
            o[6] = n.out_shape[2];
            o[7] = n.kernel[0] * 100 + n.stride[0] * 10 + n.padding[0];
            double ws = 0, bs = 0;
            const size_t nw = shim_nodes[i]->weights().size(), nb = shim_nodes[i]->biases().size();
            for (size_t q = 0; q < nw; ++q) ws += n.weight[q];
            for (size_t q = 0; q < nb; ++q) bs += n.bias[q];
            o[8] = ws;
            o[9] = bs;
            o[10] = (double)nw;
            o[11] = n.scale;
        }
        return 0;
    } catch (const std::exception& e) {
        set_error(err, errlen, e.what());
        return 1;
    }
}

}  // extern "C"
