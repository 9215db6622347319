// luna_b200_shim.cpp -- see luna_b200_shim.h.
#include "luna_b200_shim.h"

#include <cstring>
#include <stdexcept>
#include <variant>

namespace lb200_luna {

namespace {

void check(int rc, const char* what) {
    if (rc != 0) {
        char msg[2048] = {0};
        lb200_last_error(msg, sizeof msg);
        throw std::runtime_error(std::string(what) + ": " + msg);
    }
}

std::vector<float> host_floats(const torch::Tensor& t) {
    auto c = t.detach().to(torch::kCPU, torch::kFloat32).contiguous();
    return std::vector<float>(c.data_ptr<float>(), c.data_ptr<float>() + c.numel());
}

template <class Opts>
void conv_geometry(const Opts& o, lb200_node_desc& d, bool transposed) {
    const auto& k = o.kernel_size();
    const auto& s = o.stride();
    const auto& dil = o.dilation();
    if (!std::holds_alternative<torch::ExpandingArray<2>>(o.padding()))
        throw std::runtime_error("lb200_luna: 'same' / 'valid' conv padding is not supported");
    const auto& p = std::get<torch::ExpandingArray<2>>(o.padding());
    if (o.groups() != 1 || (*dil)[0] != 1 || (*dil)[1] != 1)
        throw std::runtime_error("lb200_luna: grouped or dilated convolutions are not supported");
    for (int i = 0; i < 2; ++i) {
        d.kernel[i] = (int32_t)(*k)[i];
        d.stride[i] = (int32_t)(*s)[i];
        d.padding[i] = (int32_t)(*p)[i];
        d.output_padding[i] = transposed ? (int32_t)(*o.output_padding())[i] : 0;
    }
}

}  // namespace

// ------------------------------------------------------------ nodes
BoundedNode::BoundedNode(NLR::NodeType t) { d_.type = static_cast<int32_t>(t); }

void BoundedNode::keep(const torch::Tensor& t, std::vector<float>& dst) { dst = host_floats(t); }

void BoundedNode::setOutputShape(const std::vector<int>& shape) {
    // {1, C, H, W} as Luna's conv nodes take it, or {C, H, W}.
    const size_t o = shape.size() == 4 ? 1 : 0;
    if (shape.size() - o != 3) throw std::runtime_error("lb200_luna: output shape must be {1, C, H, W}");
    for (int i = 0; i < 3; ++i) d_.out_shape[i] = shape[o + i];
}

void BoundedNode::setOutputSize(unsigned size) {
    d_.out_shape[0] = (int32_t)size;
    d_.out_shape[1] = d_.out_shape[2] = 1;
}

unsigned BoundedNode::getOutputSize() const {
    return (unsigned)d_.out_shape[0] * (unsigned)d_.out_shape[1] * (unsigned)d_.out_shape[2];
}

BoundedInputNode::BoundedInputNode(unsigned, unsigned inputSize, const std::string&)
    : BoundedNode(NLR::NodeType::INPUT) {
    setOutputSize(inputSize);
}

BoundedLinearNode::BoundedLinearNode(const torch::nn::Linear& linear, float alpha, const std::string&)
    : BoundedNode(NLR::NodeType::LINEAR) {
    keep(linear->weight, w_);
    if (linear->bias.defined()) keep(linear->bias, b_);
    d_.in_features = linear->weight.size(1);
    d_.out_features = linear->weight.size(0);
    d_.scale = alpha;
    setOutputSize((unsigned)d_.out_features);
}

BoundedConvNode::BoundedConvNode(const torch::nn::Conv2d& conv, NLR::ConvMode, const std::string&)
    : BoundedNode(NLR::NodeType::CONV) {
    keep(conv->weight, w_);
    if (conv->bias.defined()) keep(conv->bias, b_);
    conv_geometry(conv->options, d_, false);
    d_.out_shape[0] = (int32_t)conv->weight.size(0);  // H, W: setOutputShape
}

BoundedConvTransposeNode::BoundedConvTransposeNode(const torch::nn::ConvTranspose2d& conv, NLR::ConvMode,
                                                   const std::string&)
    : BoundedNode(NLR::NodeType::CONVTRANSPOSE) {
    keep(conv->weight, w_);
    if (conv->bias.defined()) keep(conv->bias, b_);
    conv_geometry(conv->options, d_, true);
    d_.out_shape[0] = (int32_t)conv->weight.size(1);
}

BoundedBatchNormNode::BoundedBatchNormNode(const torch::Tensor& scale, const torch::Tensor& B,
                                           const torch::Tensor& mean, const torch::Tensor& var, float eps,
                                           const std::string&)
    : BoundedNode(NLR::NodeType::BATCHNORM) {
    keep(scale, w_);
    keep(B, b_);
    keep(mean, mean_);
    keep(var, var_);
    d_.eps = eps;
}

BoundedReLUNode::BoundedReLUNode(const torch::nn::ReLU&, const std::string&) : BoundedNode(NLR::NodeType::RELU) {}
BoundedSigmoidNode::BoundedSigmoidNode(const torch::nn::Sigmoid&, const std::string&)
    : BoundedNode(NLR::NodeType::SIGMOID) {}
BoundedAddNode::BoundedAddNode() : BoundedNode(NLR::NodeType::ADD) {}
BoundedFlattenNode::BoundedFlattenNode() : BoundedNode(NLR::NodeType::FLATTEN) {}
BoundedIdentityNode::BoundedIdentityNode() : BoundedNode(NLR::NodeType::IDENTITY) {}
BoundedReshapeNode::BoundedReshapeNode() : BoundedNode(NLR::NodeType::RESHAPE) {}
BoundedSubNode::BoundedSubNode() : BoundedNode(NLR::NodeType::SUB) { d_.constant_second = 1; }

void BoundedSubNode::setConstantValue(const torch::Tensor& constant, bool isSecondOperand) {
    keep(constant, const_);
    d_.constant_second = isSecondOperand ? 1 : 0;
}

BoundedSliceNode::BoundedSliceNode(int64_t start, int64_t end, int64_t axes, int64_t steps, const std::string&)
    : BoundedNode(NLR::NodeType::SLICE) {
    d_.start = start;
    d_.end = end;
    d_.axis = (int32_t)axes;
    d_.step = steps;
}

BoundedConcatNode::BoundedConcatNode(int axis, unsigned, const std::string&) : BoundedNode(NLR::NodeType::CONCAT) {
    d_.axis = axis;
}

// ------------------------------------------------------------ model
TorchModel::TorchModel(const std::vector<std::shared_ptr<BoundedNode>>& nodes,
                       const std::vector<unsigned>& inputIndices, unsigned outputIndex,
                       const std::map<unsigned, std::vector<unsigned>>& dependencies, int device)
    : nodes_(nodes) {
    if (inputIndices.size() != 1) throw std::runtime_error("lb200_luna: exactly one input node is supported");
    const int n = (int)nodes.size();
    descs_.resize(n);
    for (int i = 0; i < n; ++i) {
        if (!nodes[i]) throw std::runtime_error("lb200_luna: null node " + std::to_string(i));
        descs_[i] = nodes[i]->desc();
        auto it = dependencies.find((unsigned)i);
        const std::vector<unsigned> deps = it == dependencies.end() ? std::vector<unsigned>{} : it->second;
        if (deps.size() > 4) throw std::runtime_error("lb200_luna: more than 4 dependencies");
        descs_[i].num_inputs = (int32_t)deps.size();
        for (size_t k = 0; k < deps.size(); ++k) descs_[i].inputs[k] = (int32_t)deps[k];
    }
    // Shapes not given explicitly follow the producer, as a forward pass
    // would size them (element-wise nodes keep it, Flatten flattens it).
    for (int i = 0; i < n; ++i) {
        lb200_node_desc& d = descs_[i];
        const bool has = d.out_shape[0] > 0 && d.out_shape[1] > 0 && d.out_shape[2] > 0;
        if (has || d.num_inputs == 0) continue;
        if (d.inputs[0] >= i) throw std::runtime_error("lb200_luna: nodes must be in topological order");
        const lb200_node_desc& p = descs_[d.inputs[0]];
        if (d.type == LB200_NODE_FLATTEN || d.type == LB200_NODE_RESHAPE) {
            d.out_shape[0] = p.out_shape[0] * p.out_shape[1] * p.out_shape[2];
            d.out_shape[1] = d.out_shape[2] = 1;
        } else if (d.type == LB200_NODE_CONV || d.type == LB200_NODE_CONVTRANSPOSE || d.type == LB200_NODE_SLICE ||
                   d.type == LB200_NODE_CONCAT) {
            throw std::runtime_error("lb200_luna: node " + std::to_string(i) + " needs setOutputShape / setOutputSize");
        } else {
            for (int k = 0; k < 3; ++k) d.out_shape[k] = p.out_shape[k];
        }
    }
    // Host pointers into the nodes' copies (read once by lb200_model_create).
    for (int i = 0; i < n; ++i) {
        const auto& node = *nodes_[i];
        lb200_node_desc& d = descs_[i];
        d.weight = node.weights().empty() ? nullptr : node.weights().data();
        d.bias = node.biases().empty() ? nullptr : node.biases().data();
        d.running_mean = node.means().empty() ? nullptr : node.means().data();
        d.running_var = node.vars().empty() ? nullptr : node.vars().data();
        d.constant = node.constants().empty() ? nullptr : node.constants().data();
    }
    lb200_graph_desc& g = graph_;
    g.num_nodes = n;
    g.nodes = descs_.data();
    g.input_index = (int32_t)inputIndices[0];
    g.output_index = (int32_t)outputIndex;
    const lb200_node_desc& din = descs_[g.input_index];
    const lb200_node_desc& dout = descs_[g.output_index];
    n_in_ = (unsigned)din.out_shape[0] * din.out_shape[1] * din.out_shape[2];
    n_out_ = (unsigned)dout.out_shape[0] * dout.out_shape[1] * dout.out_shape[2];
    if (device >= 0) check(lb200_model_create(&g, device, &model_), "lb200_model_create");
}

std::string TorchModel::describe() const {
    size_t need = 0;
    check(lb200_describe_plan(&graph_, nullptr, nullptr, 0, &need), "lb200_describe_plan");
    std::string buf(need, '\0');
    check(lb200_describe_plan(&graph_, nullptr, buf.data(), need, &need), "lb200_describe_plan");
    buf.resize(std::strlen(buf.c_str()));
    return buf;
}

TorchModel::~TorchModel() {
    if (model_) lb200_model_destroy(model_);
}

void TorchModel::setInputBounds(const BoundedTensor<torch::Tensor>& inputBounds) { input_ = inputBounds; }

void TorchModel::setSpecificationMatrix(const torch::Tensor& specMatrix) { C_ = specMatrix; }

BoundedTensor<torch::Tensor> TorchModel::compute_bounds(const BoundedTensor<torch::Tensor>& input_bounds,
                                                        const torch::Tensor* specification_matrix,
                                                        LunaConfiguration::AnalysisMethod method, bool bound_lower,
                                                        bool bound_upper) {
    setInputBounds(input_bounds);
    if (specification_matrix) setSpecificationMatrix(*specification_matrix);
    // TorchModel.cpp:668-698: the method and the computed sides are
    // recorded in the configuration; alpha-CROWN optimises a side only when
    // it is computed and its OPTIMIZE_* flag is set.
    LunaConfiguration::ANALYSIS_METHOD = method;
    LunaConfiguration::COMPUTE_LOWER = bound_lower;
    LunaConfiguration::COMPUTE_UPPER = bound_upper;
    if (method == LunaConfiguration::AnalysisMethod::CROWN) return runCROWN(input_bounds);
    return runAlphaCROWN(input_bounds, bound_lower && LunaConfiguration::OPTIMIZE_LOWER,
                         bound_upper && LunaConfiguration::OPTIMIZE_UPPER);
}

BoundedTensor<torch::Tensor> TorchModel::runCROWN(const BoundedTensor<torch::Tensor>& inputBounds) {
    return run(inputBounds, LB200_METHOD_CROWN, LunaConfiguration::COMPUTE_LOWER, LunaConfiguration::COMPUTE_UPPER,
               false, false);
}

BoundedTensor<torch::Tensor> TorchModel::runAlphaCROWN(const BoundedTensor<torch::Tensor>& inputBounds,
                                                       bool optimizeLower, bool optimizeUpper) {
    return run(inputBounds, LB200_METHOD_ALPHA_CROWN, LunaConfiguration::COMPUTE_LOWER,
               LunaConfiguration::COMPUTE_UPPER, optimizeLower, optimizeUpper);
}

BoundedTensor<torch::Tensor> TorchModel::run(const BoundedTensor<torch::Tensor>& in, int method, bool lower,
                                             bool upper, bool opt_lower, bool opt_upper) {
    // Input bounds: flat [n] as Luna takes them, or [B, n] for a batch.
    auto xl = in.lower().detach().to(torch::kCPU, torch::kFloat32).contiguous();
    auto xu = in.upper().detach().to(torch::kCPU, torch::kFloat32).contiguous();
    if (xl.numel() % n_in_ != 0 || xl.numel() != xu.numel())
        throw std::runtime_error("lb200_luna: input bounds do not match the input size");
    const int64_t B = xl.numel() / n_in_;
    // Specification C [nspec, 1, n_out] (Luna) or the identity (bounds of every output).
    torch::Tensor C = C_.defined() ? C_.detach().to(torch::kCPU, torch::kFloat32).reshape({-1, (int64_t)n_out_})
                                   : torch::eye(n_out_, torch::kFloat32);
    C = C.contiguous();
    const int64_t nspec = C.size(0);
    lb200_options o{};
    lb200_options_default(&o);
    o.alpha_iterations = LunaConfiguration::ALPHA_ITERATIONS;
    o.alpha_lr = LunaConfiguration::ALPHA_LR;
    o.alpha_lr_decay = LunaConfiguration::ALPHA_LR_DECAY;
    o.early_stop_patience = LunaConfiguration::EARLY_STOP_PATIENCE;
    o.start_save_best = LunaConfiguration::START_SAVE_BEST;
    o.stabilize_intermediate_bounds = LunaConfiguration::STABILIZE_INTERMEDIATE_BOUNDS;
    o.recompute_intermediate_bounds = LunaConfiguration::RECOMPUTE_INTERMEDIATE_BOUNDS;
    o.optimize_lower = opt_lower;
    o.optimize_upper = opt_upper;
    o.stop_crown_on_verified = LunaConfiguration::STOP_CROWN_ON_VERIFIED;
    o.stop_alpha_on_verified = LunaConfiguration::STOP_ALPHA_ON_VERIFIED;
    o.enable_first_linear_ibp = LunaConfiguration::ENABLE_FIRST_LINEAR_IBP;
    o.use_patches_mode = LunaConfiguration::USE_PATCHES_MODE;
    if (!model_) throw std::runtime_error("lb200_luna: a host-only model (device < 0) cannot bound");
    check(lb200_set_options(model_, &o), "lb200_set_options");
    auto lb = torch::zeros({B, nspec}, torch::kFloat32);
    auto ub = torch::zeros({B, nspec}, torch::kFloat32);
    check(lb200_compute_bounds(model_, method, xl.data_ptr<float>(), xu.data_ptr<float>(), B, C.data_ptr<float>(), 1,
                               nspec, nullptr, lower, upper, lb.data_ptr<float>(), ub.data_ptr<float>(), nullptr),
          "lb200_compute_bounds");
    if (B == 1 && in.lower().dim() <= 1) {
        lb = lb.reshape({nspec});
        ub = ub.reshape({nspec});
    }
    final_ = BoundedTensor<torch::Tensor>(lb, ub);
    return final_;
}

}  // namespace lb200_luna
