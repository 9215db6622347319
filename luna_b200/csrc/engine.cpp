// engine.cpp -- host orchestration of IBP, CROWN and alpha-CROWN on a batch
// of boxes (one GPU).
//
// Luna bounds one box per call and keeps per-box state on the nodes.  Here a
// chunk of B boxes shares the network weights and every backward start
// stacks the rows of all boxes: the A matrix of start s is [2 R_s, n] with
// R_s = sum over boxes of the IBP-unstable neurons of pre-activation s
// (CROWNAnalysis::computeIntermediateBoundsLazy, CROWNAnalysis.cpp:1744-1795),
// so each Linear step is a single GEMM whose epilogue applies the ReLU
// relaxation of the box that owns the row.
#include "engine.h"
#include "graph_canon.h"
#include "tc_gemm.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace lb200 {

// ------------------------------------------------------------ DevCache
DevCache::~DevCache() { release(); }

void* DevCache::get(const std::string& name, size_t bytes) {
    if (bytes == 0) bytes = 16;
    Buf& b = bufs_[name];
    if (b.bytes < bytes) {
        if (b.p) LB_CUDA(cudaFree(b.p));
        b.p = nullptr;
        const size_t want = (bytes + 255) & ~size_t(255);
        LB_CUDA(cudaMalloc(&b.p, want));
        b.bytes = want;
    }
    return b.p;
}

size_t DevCache::capacity(const std::string& name) const {
    auto it = bufs_.find(name);
    return it == bufs_.end() ? 0 : it->second.bytes;
}

size_t DevCache::total_bytes() const {
    size_t t = 0;
    for (auto& kv : bufs_) t += kv.second.bytes;
    return t;
}

void DevCache::release() {
    for (auto& kv : bufs_)
        if (kv.second.p) cudaFree(kv.second.p);
    bufs_.clear();
}

// ------------------------------------------------------------ Model
namespace {
// One input of a pre-activation: the output of level `src` (its ReLU, or the
// input for level 0) through an affine node (with a BatchNorm folded in), or
// directly (an Add operand that is an activation: an identity skip).
struct EdgeDesc {
    int src = -1;
    int affine = -1;  // node id, -1: identity
    int bn = -1;      // BatchNorm node folded into the affine node, or -1
};
// What a node's output is: an activation (level) or a sum of edges not yet
// consumed by a ReLU.
struct ValDesc {
    int kind = 0;  // 0: unsupported, 1: activation of `level`, 2: pre-activation sum
    int level = -1;
    std::vector<EdgeDesc> edges;
};
}  // namespace

// The graph must be Luna's feed-forward verification nets: an input, then
// pre-activations each feeding one ReLU, each pre-activation the sum of an
// affine map (Linear / Conv2d / ConvTranspose2d, optionally followed by
// BatchNorm) of the level just below and, through an Add
// (BoundedAddNode, two tensor operands), of skip edges from earlier levels
// (the activation itself, or a conv of it); the output is a Linear of the
// last level.  Flatten and Identity nodes pass through.
Model::Model(const lb200_graph_desc* g_in, int device, bool on_device) : device_(device), on_device_(on_device) {
    if (!g_in || g_in->num_nodes <= 0 || !g_in->nodes) throw std::invalid_argument("empty graph");
    if (on_device_) LB_CUDA(cudaSetDevice(device_));
    // Reshape / Sub / Slice / Concat restated as the affine kinds below
    // (graph_canon.h); nodes left without a path to the output are skipped.
    const CanonGraph cg = canonicalize(g_in);
    const lb200_graph_desc* g = &cg.desc;
    const int n = g->num_nodes;
    std::vector<std::vector<int>> dependents(n);
    std::vector<int> indeg(n, 0);
    for (int i = 0; i < n; ++i) {
        if (cg.dead[i]) continue;
        const auto& d = g->nodes[i];
        if (d.num_inputs < 0 || d.num_inputs > 4) throw std::invalid_argument("bad num_inputs");
        for (int k = 0; k < d.num_inputs; ++k) {
            if (d.inputs[k] < 0 || d.inputs[k] >= n) throw std::invalid_argument("bad input index");
            dependents[d.inputs[k]].push_back(i);
        }
        indeg[i] = d.num_inputs;
    }
    if (g->input_index < 0 || g->input_index >= n || g->nodes[g->input_index].type != LB200_NODE_INPUT)
        throw std::invalid_argument("input_index must name an INPUT node");
    if (g->output_index < 0 || g->output_index >= n) throw std::invalid_argument("bad output_index");
    // Topological order (Kahn, ties by node id: TorchModel::topologicalSort).
    std::vector<int> order;
    {
        std::vector<int> q;
        int live = 0;
        for (int i = 0; i < n; ++i) {
            if (cg.dead[i]) continue;
            ++live;
            if (indeg[i] == 0) q.push_back(i);
        }
        for (size_t h = 0; h < q.size(); ++h) {
            order.push_back(q[h]);
            for (int d : dependents[q[h]])
                if (--indeg[d] == 0) q.push_back(d);
        }
        if ((int)order.size() != live) throw std::invalid_argument("graph has a cycle");
    }
    auto bad = [&](int i, const std::string& why) {
        throw std::invalid_argument("node " + std::to_string(i) + " (type " + std::to_string(g->nodes[i].type) +
                                    "): " + why);
    };
    std::vector<ValDesc> val(n);
    std::vector<std::vector<EdgeDesc>> lvl_edges(1);  // level 0 = input
    std::vector<int> lvl_node(1, g->input_index);     // node whose output is the level's pre-activation
    std::vector<int> lvl_act(1, 0);                   // activation of each level (0: none)
    for (int i : order) {
        const auto& d = g->nodes[i];
        ValDesc& v = val[i];
        auto operand = [&](int k) -> const ValDesc& { return val[d.inputs[k]]; };
        switch (d.type) {
        case LB200_NODE_INPUT:
            if (i != g->input_index) bad(i, "a second input node");
            v.kind = 1;
            v.level = 0;
            break;
        case LB200_NODE_FLATTEN:
        case LB200_NODE_IDENTITY:
            if (d.num_inputs != 1) bad(i, "expects one input");
            v = operand(0);
            break;
        case LB200_NODE_LINEAR:
        case LB200_NODE_CONV:
        case LB200_NODE_CONVTRANSPOSE:
            if (d.num_inputs != 1 || operand(0).kind != 1)
                bad(i, "an affine node must take the input or a ReLU output");
            if (!d.weight) bad(i, "affine node without weight");
            v.kind = 2;
            v.edges = {EdgeDesc{operand(0).level, i, -1}};
            break;
        case LB200_NODE_BATCHNORM:
            // Folded into the affine node before it (an affine map of an affine
            // map; BoundedBatchNormNode.cpp:68-80,180-532).
            if (d.num_inputs != 1 || operand(0).kind != 2 || operand(0).edges.size() != 1 ||
                operand(0).edges[0].affine < 0 || operand(0).edges[0].bn >= 0)
                bad(i, "BatchNorm must directly follow a Linear or Conv node");
            if (!d.weight || !d.bias || !d.running_mean || !d.running_var) bad(i, "BatchNorm without parameters");
            v = operand(0);
            v.edges[0].bn = i;
            break;
        case LB200_NODE_ADD:
            // BoundedAddNode of two tensors (:167-279): A reaches both operands.
            if (d.num_inputs != 2) bad(i, "Add with a constant operand is not supported");
            v.kind = 2;
            for (int k = 0; k < 2; ++k) {
                const ValDesc& o = operand(k);
                if (o.kind == 1)
                    v.edges.push_back(EdgeDesc{o.level, -1, -1});
                else if (o.kind == 2)
                    v.edges.insert(v.edges.end(), o.edges.begin(), o.edges.end());
                else
                    bad(i, "unsupported Add operand");
            }
            break;
        case LB200_NODE_RELU:
        case LB200_NODE_SIGMOID:
            if (d.num_inputs != 1 || operand(0).kind != 2)
                bad(i, "an activation must follow an affine node or an Add");
            lvl_edges.push_back(operand(0).edges);
            lvl_node.push_back(d.inputs[0]);
            lvl_act.push_back(d.type == LB200_NODE_SIGMOID ? ACT_SIGMOID : ACT_RELU);
            v.kind = 1;
            v.level = (int)lvl_edges.size() - 1;
            break;
        default:
            bad(i, "node kind not supported by this engine build");
        }
        // A pre-activation sum is consumed exactly once (by its ReLU, an Add,
        // a BatchNorm or as the output).
        if (v.kind == 2 && i != g->output_index && dependents[i].size() != 1)
            bad(i, "a pre-activation used by several nodes");
    }
    if (val[g->output_index].kind != 2) throw std::invalid_argument("the output node must be an affine node");
    lvl_edges.push_back(val[g->output_index].edges);
    lvl_node.push_back(g->output_index);
    lvl_act.push_back(0);
    act_ = lvl_act;
    K_ = (int)lvl_edges.size() - 1;
    if (K_ < 2) throw std::invalid_argument("need at least two affine layers");
    // Main edge of every level: the affine edge from the level just below.
    layers_.resize(K_);
    skips_.assign(K_ + 1, {});
    std::vector<EdgeDesc> main_edge(K_ + 1);
    for (int m = 1; m <= K_; ++m) {
        bool found = false;
        for (const EdgeDesc& e : lvl_edges[m]) {
            if (!found && e.src == m - 1 && e.affine >= 0) {
                main_edge[m] = e;
                found = true;
                continue;
            }
            if (e.src < 1 || e.src > m - 2)
                throw std::invalid_argument("level " + std::to_string(m) +
                                            ": a skip edge must come from a ReLU output at least two levels below");
            SkipEdge s;
            s.src = e.src;
            s.node = e.affine;
            s.bn = e.bn;
            skips_[m].push_back(s);
        }
        if (!found)
            throw std::invalid_argument("level " + std::to_string(m) +
                                        ": no affine input from the level below (unsupported graph shape)");
    }
    for (int m = 1; m < K_; ++m) preact_node_ids_.push_back(lvl_node[m]);
    if (g->nodes[main_edge[K_].affine].type != LB200_NODE_LINEAR || main_edge[K_].bn >= 0 || !skips_[K_].empty())
        throw std::invalid_argument("the output node must be a Linear of the last ReLU");

    const auto& din = g->nodes[g->input_index];
    MapShape in0;
    in0.C = din.out_shape[0];
    in0.H = std::max(1, din.out_shape[1]);
    in0.W = std::max(1, din.out_shape[2]);
    const int t1 = g->nodes[main_edge[1].affine].type;
    in0.spatial = t1 == LB200_NODE_CONV || t1 == LB200_NODE_CONVTRANSPOSE;
    if (!in0.spatial) in0 = MapShape{in0.n(), 1, 1, false};
    for (int m = 1; m <= K_; ++m) {
        const MapShape& prev = m == 1 ? in0 : layers_[m - 2].out;
        build_layer(layers_[m - 1], g, main_edge[m].affine, main_edge[m].bn, prev, m - 1, m == 1);
        for (size_t e = 0; e < skips_[m].size(); ++e) {
            SkipEdge& s = skips_[m][e];
            const MapShape& src = layers_[s.src - 1].out;
            const MapShape& dst = layers_[m - 1].out;
            if (s.node >= 0) {
                if (g->nodes[s.node].type != LB200_NODE_CONV)
                    throw std::invalid_argument("a skip edge through an affine node must be a Conv2d");
                s.L = std::make_shared<Layer>();
                build_layer(*s.L, g, s.node, s.bn, src, 1000 + 8 * m + (int)e, false);
                if (s.L->out.C != dst.C || s.L->out.H != dst.H || s.L->out.W != dst.W)
                    throw std::invalid_argument("level " + std::to_string(m) + ": Add operands differ in shape");
            } else if (src.C != dst.C || src.H != dst.H || src.W != dst.W || src.spatial != dst.spatial) {
                throw std::invalid_argument("level " + std::to_string(m) + ": Add operands differ in shape");
            }
            // The skip's source must be relaxed by a conv step (its addend
            // joins that step's relaxation epilogue).
            if (!layers_[s.src].conv)
                throw std::invalid_argument("a skip source must feed a Conv2d on the main path");
            if (layers_[m - 1].convt) throw std::invalid_argument("an Add after a transposed conv is not supported");
        }
    }
    if (layers_[K_ - 1].conv) throw std::invalid_argument("the output layer must be Linear");
    // Sigmoid levels: flat maps relaxed by the Linear above them.
    for (int m = 1; m < K_; ++m) {
        if (act_[m] != ACT_SIGMOID) continue;
        has_sigmoid_ = true;
        if (map(m).spatial || layers_[m].conv || layers_[m].convt)
            throw std::invalid_argument("a Sigmoid is supported on flat (Linear) layers only");
        for (int t = m + 2; t <= K_; ++t)
            for (const SkipEdge& sk : skips_[t])
                if (sk.src == m) throw std::invalid_argument("a Sigmoid output as a skip source is not supported");
    }
    // Bias that the back-substitution adds for level m: the main edge's (none
    // for a ConvTranspose: Luna's A is flat there) plus every skip conv's.
    lvl_b_.assign(K_ + 1, nullptr);
    lvl_bn_.assign(K_ + 1, nullptr);
    for (int m = 1; m <= K_; ++m) {
        const Layer& L = layers_[m - 1];
        if (L.convt) continue;
        if (skips_[m].empty()) {
            lvl_b_[m] = L.b;
            lvl_bn_[m] = L.b_neuron;
            continue;
        }
        const int nc = L.conv ? L.out.C : L.n_out;
        std::vector<float> b(L.b_host), bn((size_t)L.n_out);
        for (const SkipEdge& s : skips_[m]) {
            if (!s.L) continue;
            for (int c = 0; c < nc; ++c) b[c] += s.L->b_host[c];
        }
        for (int j = 0; j < L.n_out; ++j) bn[j] = b[j % nc];
        if (!on_device_) continue;
        lvl_b_[m] = weights_.as<float>(key("lvlb", m), b.size());
        lvl_bn_[m] = weights_.as<float>(key("lvlbn", m), bn.size());
        LB_CUDA(cudaMemcpy(lvl_b_[m], b.data(), b.size() * 4, cudaMemcpyHostToDevice));
        LB_CUDA(cudaMemcpy(lvl_bn_[m], bn.data(), bn.size() * 4, cudaMemcpyHostToDevice));
    }
    build_geometry();
    lb200_options_default(&opt_);
    if (cg.in_tf) {
        in_tf_ = true;
        in_neg_ = cg.in_neg;
        if ((int)cg.in_const.size() != width(0)) throw std::invalid_argument("input Sub constant size");
        if (on_device_) {
            in_const_ = weights_.as<float>("in_const", cg.in_const.size());
            LB_CUDA(cudaMemcpy(in_const_, cg.in_const.data(), cg.in_const.size() * 4, cudaMemcpyHostToDevice));
        }
    }
}

// One affine edge: the node's weight and bias with a following BatchNorm
// folded in, laid out for the engine's kernels.
void Model::build_layer(Layer& L, const lb200_graph_desc* g, int node, int bn_node, const MapShape& prev, int k,
                        bool first) {
    const auto& d = g->nodes[node];
    L.conv = d.type == LB200_NODE_CONV;
    L.convt = d.type == LB200_NODE_CONVTRANSPOSE;
    L.in = prev;
    if (L.convt) {
        has_conv_ = true;
        if (!prev.spatial) throw std::invalid_argument("a transposed conv must follow the input or a conv");
        if (first) throw std::invalid_argument("a transposed conv as the first layer is not supported");
        if (bn_node >= 0) throw std::invalid_argument("BatchNorm after a transposed conv is not supported");
        L.kh = d.kernel[0];
        L.kw = d.kernel[1];
        L.sh = d.stride[0];
        L.sw = d.stride[1];
        L.ph = d.padding[0];
        L.pw = d.padding[1];
        if (d.output_padding[0] != 0 || d.output_padding[1] != 0)
            throw std::invalid_argument("ConvTranspose output_padding must be 0 (BoundedConvTransposeNode.cpp:61-63)");
        if (L.kh <= 0 || L.kw <= 0 || L.sh <= 0 || L.sw <= 0 || L.ph < 0 || L.pw < 0)
            throw std::invalid_argument("bad transposed-conv geometry");
        L.out.C = d.out_shape[0];
        L.out.H = (prev.H - 1) * L.sh - 2 * L.ph + L.kh;
        L.out.W = (prev.W - 1) * L.sw - 2 * L.pw + L.kw;
        L.out.spatial = true;
        if (L.out.H != d.out_shape[1] || L.out.W != d.out_shape[2] || L.out.H <= 0 || L.out.W <= 0)
            throw std::invalid_argument("transposed-conv out_shape does not match its geometry");
    } else if (L.conv) {
        has_conv_ = true;
        if (!prev.spatial) throw std::invalid_argument("a conv layer must follow the input or another conv");
        L.kh = d.kernel[0];
        L.kw = d.kernel[1];
        L.sh = d.stride[0];
        L.sw = d.stride[1];
        L.ph = d.padding[0];
        L.pw = d.padding[1];
        if (L.kh <= 0 || L.kw <= 0 || L.sh <= 0 || L.sw <= 0 || L.ph < 0 || L.pw < 0)
            throw std::invalid_argument("bad conv geometry");
        L.out.C = d.out_shape[0];
        L.out.H = (prev.H + 2 * L.ph - L.kh) / L.sh + 1;
        L.out.W = (prev.W + 2 * L.pw - L.kw) / L.sw + 1;
        L.out.spatial = true;
        if (L.out.H != d.out_shape[1] || L.out.W != d.out_shape[2])
            throw std::invalid_argument("conv out_shape does not match its geometry");
    } else {
        if (d.in_features <= 0 || d.out_features <= 0) throw std::invalid_argument("Linear node without sizes");
        if (d.in_features != prev.n()) throw std::invalid_argument("width mismatch");
        L.out = MapShape{(int)d.out_features, 1, 1, false};
    }
    L.n_in = L.in.n();
    L.n_out = L.out.n();
    const int Ci = L.in.C, Co = L.out.C;
    // The node's weight and bias with a following BatchNorm folded in:
    // y = w (affine(x)) + (B - mean w), w = scale / sqrt(var + eps) per
    // output channel (conv) or feature (Linear), computed in fp32 as
    // BoundedBatchNormNode::ensureCachedParams does (:68-80).
    const int nch = (L.conv || L.convt) ? Co : L.n_out;
    const size_t per_ch = (L.conv || L.convt) ? (size_t)Ci * L.kh * L.kw : (size_t)L.n_in;
    std::vector<float> wsrc(d.weight, d.weight + (size_t)nch * per_ch), bsrc(nch, 0.f);
    if (d.bias)
        for (int c = 0; c < nch; ++c) bsrc[c] = d.bias[c];
    if (bn_node >= 0) {
        const auto& nb = g->nodes[bn_node];
        for (int c = 0; c < nch; ++c) {
            const float w = nb.weight[c] / std::sqrt(nb.running_var[c] + nb.eps);
            for (size_t q = 0; q < per_ch; ++q) wsrc[(size_t)c * per_ch + q] *= w;
            bsrc[c] = bsrc[c] * w + (nb.bias[c] - nb.running_mean[c] * w);
        }
    }
    std::vector<float> W, Wt, b(bsrc), bn(L.n_out, 0.f);
    if (L.convt) {
        // ONNX ConvTranspose weight [Ci, Co, kh, kw] -> Wg [Ci][kh][kw][Co], Wa [kh][kw][Co][Ci].
        W.resize((size_t)Ci * L.kh * L.kw * Co);
        Wt.resize(W.size());
        for (int c = 0; c < Ci; ++c)
            for (int o = 0; o < Co; ++o)
                for (int y = 0; y < L.kh; ++y)
                    for (int x = 0; x < L.kw; ++x) {
                        const float w = wsrc[(((size_t)c * Co + o) * L.kh + y) * L.kw + x];
                        W[(((size_t)c * L.kh + y) * L.kw + x) * Co + o] = w;
                        Wt[(((size_t)y * L.kw + x) * Co + o) * Ci + c] = w;
                    }
        for (int j = 0; j < L.n_out; ++j) bn[j] = b[j % Co];
    } else if (L.conv) {
        // ONNX Conv weight [Co, Ci, kh, kw] -> Wc [Co][kh][kw][Ci], Wk [kh][kw][Co][Ci].
        W.resize((size_t)Co * L.kh * L.kw * Ci);
        Wt.resize(W.size());
        for (int o = 0; o < Co; ++o)
            for (int c = 0; c < Ci; ++c)
                for (int y = 0; y < L.kh; ++y)
                    for (int x = 0; x < L.kw; ++x) {
                        const float w = wsrc[(((size_t)o * Ci + c) * L.kh + y) * L.kw + x];
                        W[(((size_t)o * L.kh + y) * L.kw + x) * Ci + c] = w;
                        Wt[(((size_t)y * L.kw + x) * Co + o) * Ci + c] = w;
                    }
        for (int j = 0; j < L.n_out; ++j) bn[j] = b[j % Co];
    } else {
        W.resize((size_t)L.n_out * L.n_in);
        Wt.resize(W.size());
        const int HW = L.in.H * L.in.W;
        for (int o = 0; o < L.n_out; ++o)
            for (int i = 0; i < L.n_in; ++i) {
                // Input feature i in the engine's order; Luna's column is
                // its CHW index when the input is a flattened conv map.
                const int col = L.in.spatial ? (i % Ci) * HW + i / Ci : i;
                // BoundedLinearNode bakes alpha (Gemm scale) into the weight (:91-93).
                const float w = d.scale * wsrc[(size_t)o * L.n_in + col];
                W[(size_t)o * L.n_in + i] = w;
                Wt[(size_t)i * L.n_out + o] = w;
            }
        bn = b;
    }
    L.b_host = b;
    if (!on_device_) return;
    L.W = weights_.as<float>(key("W", k), W.size());
    L.Wt = weights_.as<float>(key("Wt", k), Wt.size());
    L.b = weights_.as<float>(key("b", k), b.size());
    L.b_neuron = weights_.as<float>(key("bn", k), bn.size());
    LB_CUDA(cudaMemcpy(L.W, W.data(), W.size() * 4, cudaMemcpyHostToDevice));
    LB_CUDA(cudaMemcpy(L.Wt, Wt.data(), Wt.size() * 4, cudaMemcpyHostToDevice));
    LB_CUDA(cudaMemcpy(L.b, b.data(), b.size() * 4, cudaMemcpyHostToDevice));
    LB_CUDA(cudaMemcpy(L.b_neuron, bn.data(), bn.size() * 4, cudaMemcpyHostToDevice));
    if (L.conv && k < 1000) build_tc_conv(L, wsrc.data(), k);
    if (L.convt && k < 1000) build_tc_convt(L, wsrc.data(), k);
    if (!L.conv && !L.convt) {
        L.W_hi = weights_.as<float>(key("Whi", k), W.size());
        L.W_lo = weights_.as<float>(key("Wlo", k), W.size());
        L.Wt_hi = weights_.as<float>(key("Wthi", k), Wt.size());
        L.Wt_lo = weights_.as<float>(key("Wtlo", k), Wt.size());
        launch_split_tf32(L.W, L.W_hi, L.W_lo, (int64_t)W.size(), 0);
        launch_split_tf32(L.Wt, L.Wt_hi, L.Wt_lo, (int64_t)Wt.size(), 0);
    }
    LB_CUDA(cudaDeviceSynchronize());
}

// Window of a conv's input map that the transposed conv of window `w` (on
// its output map) covers: the receptive field, (w - 1) s + k wide.
static WinGeo conv_input_window(const WinGeo& w, const Layer& L) {
    WinGeo v = w;
    v.C = L.in.C;
    v.H = L.in.H;
    v.W = L.in.W;
    if (w.full) {
        v.wh = L.in.H;
        v.ww = L.in.W;
        return v;
    }
    v.wh = (w.wh - 1) * L.sh + L.kh;
    v.ww = (w.ww - 1) * L.sw + L.kw;
    v.mul_y *= L.sh;
    v.mul_x *= L.sw;
    v.off_y = w.off_y * L.sh - L.ph;
    v.off_x = w.off_x * L.sw - L.pw;
    return v;
}

// Row geometry of every start at every level up to it: receptive-field
// windows for a conv start with only convs (and identity / conv skips)
// below it, whole maps otherwise.  A skip's window must lie inside the main
// path's window at its source level (true for "same"-padded blocks and 1x1
// projections).
void Model::build_geometry() {
    geo_.assign(K_ + 1, {});
    for (int st = 2; st <= K_; ++st) {
        std::vector<WinGeo>& gv = geo_[st];
        gv.resize(st + 1);
        bool window = st < K_ && layers_[st - 1].conv;
        for (int m = st; m >= 1 && window; --m) {
            window = layers_[m - 1].conv;
            for (const SkipEdge& s : skips_[m]) window = window && (!s.L || s.L->conv);
        }
        for (int m = 0; m <= st; ++m) {
            const MapShape& ms = map(m);
            WinGeo w;
            w.C = ms.C;
            w.H = ms.H;
            w.W = ms.W;
            w.wh = ms.H;
            w.ww = ms.W;
            gv[m] = w;
        }
        if (!window) continue;
        // The start row itself: one pixel of the start map.
        WinGeo& ws = gv[st];
        ws.full = 0;
        ws.wh = ws.ww = 1;
        ws.mul_y = ws.mul_x = 1;
        ws.off_y = ws.off_x = 0;
        ws.st_C = map(st).C;
        ws.st_W = map(st).W;
        for (int m = st; m >= 1; --m) gv[m - 1] = conv_input_window(gv[m], layers_[m - 1]);
        for (int m = st; m >= 2; --m)
            for (const SkipEdge& s : skips_[m]) {
                const WinGeo w = s.L ? conv_input_window(gv[m], *s.L) : gv[m];
                const WinGeo& o = gv[s.src];
                if (w.mul_y != o.mul_y || w.mul_x != o.mul_x || w.off_y < o.off_y || w.off_x < o.off_x ||
                    w.off_y + w.wh > o.off_y + o.wh || w.off_x + w.ww > o.off_x + o.ww)
                    throw std::invalid_argument("level " + std::to_string(m) +
                                                ": a skip edge reaches outside the main path's window");
            }
    }
}

// Weight matrices of the tensor-core conv steps of one conv layer.
void Model::build_tc_conv(Layer& L, const float* w, int k) {
    const int Co = L.out.C, Ci = L.in.C, kh = L.kh, kw = L.kw, s = L.sh;
    if (L.sh != L.sw) return;
    auto wv = [&](int co, int ci, int ky, int kx) { return w[(((size_t)co * Ci + ci) * kh + ky) * kw + kx]; };
    L.Uy = (kh + s - 1) / s;
    L.Ux = (kw + s - 1) / s;
    if (Co % 32 == 0 && s * s * Ci >= 64 && L.Uy * L.Ux * (Co / 32) <= TC_CONV_MAX_KB) {
        const int mt = s * s * Ci, kt = L.Uy * L.Ux * Co;
        std::vector<float> Wf((size_t)mt * kt, 0.f);
        for (int py = 0; py < s; ++py)
            for (int px = 0; px < s; ++px)
                for (int ci = 0; ci < Ci; ++ci)
                    for (int uy = 0; uy < L.Uy; ++uy)
                        for (int ux = 0; ux < L.Ux; ++ux) {
                            const int ky = py + s * uy, kx = px + s * ux;
                            if (ky >= kh || kx >= kw) continue;
                            for (int co = 0; co < Co; ++co)
                                Wf[(size_t)((py * s + px) * Ci + ci) * kt + (uy * L.Ux + ux) * Co + co] =
                                    wv(co, ci, ky, kx);
                        }
        float* tmp = weights_.as<float>(key("Wf", k), Wf.size());
        LB_CUDA(cudaMemcpy(tmp, Wf.data(), Wf.size() * 4, cudaMemcpyHostToDevice));
        L.Wf_hi = weights_.as<float>(key("Wfhi", k), Wf.size());
        L.Wf_lo = weights_.as<float>(key("Wflo", k), Wf.size());
        launch_split_tf32(tmp, L.Wf_hi, L.Wf_lo, (int64_t)Wf.size(), 0);
        L.tcf = true;
    }
    if (Ci % 32 == 0) {
        for (int py = 0; py < s; ++py)
            for (int px = 0; px < s; ++px)
                for (int uy = 0; uy < L.Uy; ++uy)
                    for (int ux = 0; ux < L.Ux; ++ux) {
                        if (py + s * uy >= kh || px + s * ux >= kw) continue;
                        for (int cb = 0; cb < Ci / 32; ++cb) {
                            TcConvTap t;
                            t.plane = py * s + px;
                            t.dy = uy;
                            t.dx = ux;
                            t.c0 = cb * 32;
                            L.adj_kb.push_back(t);
                        }
                    }
        const int nka = (int)L.adj_kb.size();
        if (nka <= TC_CONV_MAX_KB) {
            std::vector<float> Wa((size_t)Co * nka * 32, 0.f);
            for (int a = 0; a < nka; ++a) {
                const TcConvTap& t = L.adj_kb[a];
                const int ky = t.plane / s + s * t.dy, kx = t.plane % s + s * t.dx;
                for (int co = 0; co < Co; ++co)
                    for (int cc = 0; cc < 32; ++cc)
                        Wa[(size_t)co * nka * 32 + a * 32 + cc] = wv(co, t.c0 + cc, ky, kx);
            }
            float* tmp = weights_.as<float>(key("Wa", k), Wa.size());
            LB_CUDA(cudaMemcpy(tmp, Wa.data(), Wa.size() * 4, cudaMemcpyHostToDevice));
            L.Wa_hi = weights_.as<float>(key("Wahi", k), Wa.size());
            L.Wa_lo = weights_.as<float>(key("Walo", k), Wa.size());
            launch_split_tf32(tmp, L.Wa_hi, L.Wa_lo, (int64_t)Wa.size(), 0);
            L.tca = true;
        } else {
            L.adj_kb.clear();
        }
    }
}

// Weight matrices of the tensor-core steps of one ConvTranspose2d layer
// (ONNX weight w [Ci][Co][kh][kw]).
void Model::build_tc_convt(Layer& L, const float* w, int k) {
    const int Ci = L.in.C, Co = L.out.C, kh = L.kh, kw = L.kw, s = L.sh;
    if (L.sh != L.sw) return;
    auto wv = [&](int ci, int co, int ky, int kx) { return w[(((size_t)ci * Co + co) * kh + ky) * kw + kx]; };
    // Back-substitution: P[q, ci] = sum over taps and co of A[q s - p + k, co] W[ci, co, k].
    if (Co % 32 == 0 && tc_conv_supported(Co, L.in.W, s) && kh * kw * (Co / 32) <= TC_CONV_MAX_KB) {
        for (int ky = 0; ky < kh; ++ky)
            for (int kx = 0; kx < kw; ++kx)
                for (int cb = 0; cb < Co / 32; ++cb) {
                    TcConvTap t;
                    t.plane = 0;
                    t.dy = ky - L.ph;
                    t.dx = kx - L.pw;
                    t.c0 = cb * 32;
                    L.tcb_kb.push_back(t);
                }
        const int nkb = (int)L.tcb_kb.size();
        std::vector<float> Wb((size_t)Ci * nkb * 32, 0.f);
        for (int a = 0; a < nkb; ++a) {
            const TcConvTap& t = L.tcb_kb[a];
            const int ky = t.dy + L.ph, kx = t.dx + L.pw;
            for (int ci = 0; ci < Ci; ++ci)
                for (int cc = 0; cc < 32; ++cc) Wb[(size_t)ci * nkb * 32 + a * 32 + cc] = wv(ci, t.c0 + cc, ky, kx);
        }
        float* tmp = weights_.as<float>(key("Wtb", k), Wb.size());
        LB_CUDA(cudaMemcpy(tmp, Wb.data(), Wb.size() * 4, cudaMemcpyHostToDevice));
        L.Wtb_hi = weights_.as<float>(key("Wtbhi", k), Wb.size());
        L.Wtb_lo = weights_.as<float>(key("Wtblo", k), Wb.size());
        launch_split_tf32(tmp, L.Wtb_hi, L.Wtb_lo, (int64_t)Wb.size(), 0);
        L.tct_b = true;
    }
    // Adjoint: Qbar[v, co] = sum of Pbar[q, ci] W[ci, co, k] over v + p = q s + k,
    // phases (v + p) mod s stacked in M, tap k = phase + s u.
    const int Uy = (kh + s - 1) / s, Ux = (kw + s - 1) / s;
    if (Ci % 32 == 0 && s * s * Co >= 64 && Uy * Ux * (Ci / 32) <= TC_CONV_MAX_KB &&
        tc_conv_supported(Ci, (L.out.W - 1 + L.pw) / s - L.pw / s + 1)) {
        const int mt = s * s * Co, kt = Uy * Ux * Ci;
        std::vector<float> Wj((size_t)mt * kt, 0.f);
        for (int py = 0; py < s; ++py)
            for (int px = 0; px < s; ++px)
                for (int co = 0; co < Co; ++co)
                    for (int uy = 0; uy < Uy; ++uy)
                        for (int ux = 0; ux < Ux; ++ux) {
                            const int ky = py + s * uy, kx = px + s * ux;
                            if (ky >= kh || kx >= kw) continue;
                            for (int ci = 0; ci < Ci; ++ci)
                                Wj[(size_t)((py * s + px) * Co + co) * kt + (uy * Ux + ux) * Ci + ci] =
                                    wv(ci, co, ky, kx);
                        }
        float* tmp = weights_.as<float>(key("Wtj", k), Wj.size());
        LB_CUDA(cudaMemcpy(tmp, Wj.data(), Wj.size() * 4, cudaMemcpyHostToDevice));
        L.Wtj_hi = weights_.as<float>(key("Wtjhi", k), Wj.size());
        L.Wtj_lo = weights_.as<float>(key("Wtjlo", k), Wj.size());
        launch_split_tf32(tmp, L.Wtj_hi, L.Wtj_lo, (int64_t)Wj.size(), 0);
        L.Uy = Uy;
        L.Ux = Ux;
        L.tct_a = true;
    }
}

TcConvPlan Model::tct_back_plan(int m, int rows, const float* data) const {
    const Layer& L = layers_[m - 1];
    TcConvPlan p;
    p.data = data;
    p.C = L.out.C;
    p.X = L.out.W;
    p.Y = L.out.H;
    p.P = 1;
    p.R = rows;
    p.ds = L.sh;
    p.ny = L.in.H;
    p.nx = L.in.W;
    for (const TcConvTap& t : L.tcb_kb) p.kb[p.nkb++] = t;
    p.w_hi = L.Wtb_hi;
    p.w_lo = L.Wtb_lo;
    p.m_total = L.in.C;
    tc_conv_tile(p, rows);
    return p;
}

TcConvPlan Model::tct_adj_plan(int m, int rows, const float* pbar) const {
    const Layer& L = layers_[m - 1];
    const int s = L.sh, tly = L.ph / s, tlx = L.pw / s;
    TcConvPlan p;
    p.data = pbar;
    p.C = L.in.C;
    p.X = L.in.W;
    p.Y = L.in.H;
    p.P = 1;
    p.R = rows;
    p.ny = (L.out.H - 1 + L.ph) / s - tly + 1;
    p.nx = (L.out.W - 1 + L.pw) / s - tlx + 1;
    for (int uy = 0; uy < L.Uy; ++uy)
        for (int ux = 0; ux < L.Ux; ++ux)
            for (int cb = 0; cb < L.in.C / 32; ++cb) {
                TcConvTap& t = p.kb[p.nkb++];
                t.plane = 0;
                t.dy = tly - uy;
                t.dx = tlx - ux;
                t.c0 = cb * 32;
            }
    p.w_hi = L.Wtj_hi;
    p.w_lo = L.Wtj_lo;
    p.m_total = s * s * L.out.C;
    tc_conv_tile(p, rows);
    return p;
}

// Phase grid of conv layer m for start st: output window pixel v of the
// level below sits at t = (v + c) div s - tlo in phase (v + c) mod s.
void Model::conv_phase(int st, int m, int& cy, int& cx, int& tlo_y, int& tlo_x, int& nty, int& ntx) const {
    const Layer& L = layers_[m - 1];
    const WinGeo& go = geo_[st][m - 1];
    cy = go.full ? L.ph : 0;
    cx = go.full ? L.pw : 0;
    tlo_y = cy / L.sh;
    tlo_x = cx / L.sw;
    nty = (go.wh - 1 + cy) / L.sh - tlo_y + 1;
    ntx = (go.ww - 1 + cx) / L.sw - tlo_x + 1;
}

TcConvPlan Model::tc_fwd_plan(int st, int m, int rows, const float* data) const {
    const Layer& L = layers_[m - 1];
    const WinGeo& gi = geo_[st][m];
    int cy, cx, tly, tlx, nty, ntx;
    conv_phase(st, m, cy, cx, tly, tlx, nty, ntx);
    TcConvPlan p;
    p.data = data;
    p.C = L.out.C;
    p.X = gi.ww;
    p.Y = gi.wh;
    p.P = 1;
    p.R = rows;
    p.ny = nty;
    p.nx = ntx;
    for (int uy = 0; uy < L.Uy; ++uy)
        for (int ux = 0; ux < L.Ux; ++ux)
            for (int cb = 0; cb < L.out.C / 32; ++cb) {
                TcConvTap& t = p.kb[p.nkb++];
                t.plane = 0;
                t.dy = tly - uy;
                t.dx = tlx - ux;
                t.c0 = cb * 32;
            }
    p.w_hi = L.Wf_hi;
    p.w_lo = L.Wf_lo;
    p.m_total = L.sh * L.sw * L.in.C;
    tc_conv_tile(p, rows);
    return p;
}

TcConvPlan Model::tc_adj_plan(int st, int m, int rows, const float* pbar) const {
    const Layer& L = layers_[m - 1];
    const WinGeo& gi = geo_[st][m];
    int cy, cx, tly, tlx, nty, ntx;
    conv_phase(st, m, cy, cx, tly, tlx, nty, ntx);
    TcConvPlan p;
    p.data = pbar;
    p.C = L.in.C;
    p.X = ntx;
    p.Y = nty;
    p.P = L.sh * L.sw;
    p.R = rows;
    p.ny = gi.wh;
    p.nx = gi.ww;
    for (const TcConvTap& a : L.adj_kb) {
        TcConvTap& t = p.kb[p.nkb++];
        t.plane = a.plane;
        t.dy = a.dy - tly;
        t.dx = a.dx - tlx;
        t.c0 = a.c0;
    }
    p.w_hi = L.Wa_hi;
    p.w_lo = L.Wa_lo;
    p.m_total = L.out.C;
    tc_conv_tile(p, rows);
    return p;
}

PhaseSplit Model::phase_split(int st, int m) const {
    const Layer& L = layers_[m - 1];
    PhaseSplit ps;
    int cy, cx, tly, tlx, nty, ntx;
    conv_phase(st, m, cy, cx, tly, tlx, nty, ntx);
    ps.s = L.sh;
    ps.C = L.in.C;
    ps.out_w = geo_[st][m - 1].ww;
    ps.cy = cy;
    ps.cx = cx;
    ps.tlo_y = tly;
    ps.tlo_x = tlx;
    ps.nty = nty;
    ps.ntx = ntx;
    ps.row_stride = (int64_t)L.sh * L.sw * nty * ntx * L.in.C;
    return ps;
}

// The transposed-conv step of conv layer m for the rows of start st.
ConvStep Model::conv_step(int st, int m) const {
    const Layer& L = layers_[m - 1];
    const WinGeo& gi = geo_[st][m];
    const WinGeo& go = geo_[st][m - 1];
    ConvStep cs;
    cs.Co = L.out.C;
    cs.Ci = L.in.C;
    cs.kh = L.kh;
    cs.kw = L.kw;
    cs.sh = L.sh;
    cs.sw = L.sw;
    cs.in_h = gi.wh;
    cs.in_w = gi.ww;
    cs.out_h = go.wh;
    cs.out_w = go.ww;
    cs.cy = go.full ? L.ph : 0;
    cs.cx = go.full ? L.pw : 0;
    cs.Wk = L.Wt;
    cs.Wc = L.W;
    return cs;
}

ConvTStep Model::convt_step(int m) const {
    const Layer& L = layers_[m - 1];
    ConvTStep ct;
    ct.Ci = L.in.C;
    ct.Co = L.out.C;
    ct.kh = L.kh;
    ct.kw = L.kw;
    ct.sh = L.sh;
    ct.sw = L.sw;
    ct.ph = L.ph;
    ct.pw = L.pw;
    ct.Hi = L.in.H;
    ct.Wi = L.in.W;
    ct.Ho = L.out.H;
    ct.Wo = L.out.W;
    ct.Wg = L.W;
    ct.Wa = L.Wt;
    return ct;
}

// Luna's CPU path starts a conv node with more than 4096 output features in
// patches mode (CROWNAnalysis.cpp:255-272) and converts the patches to a
// matrix once they are wider than a conv input (BoundedConvNode.cpp:671-694);
// the concretisation form follows (CROWNAnalysis.cpp:791-848 vs :1164-1224).
int Model::start_form(int st) const {
    // The start node: a conv (or its BatchNorm) starts in patches mode; an
    // Add start is a dense identity.
    if (st >= K_ || !layers_[st - 1].conv || !skips_[st].empty() || !opt_.use_patches_mode) return CONC_DENSE;
    if (layers_[st - 1].n_out <= 4096) return CONC_DENSE;
    if (geo_[st][st - 1].full)
        throw std::invalid_argument("a conv start above a Linear or transposed conv with more than 4096 features "
                                    "(Luna's patches mode there) is not supported");
    // (patches?, patch width) of the A reaching each level: a conv widens
    // the patch to (w - 1) s + k and turns it into a matrix once it is wider
    // than its input; joins keep patches only when every operand is patches
    // (CROWNAnalysis::addA, :1248-1355) and pad to the widest (Patches::add).
    std::vector<int> patches(st + 1, -1), width(st + 1, 0);
    patches[st] = 1;
    width[st] = 1;  // identity patches act as 1 x 1 patches
    auto join = [&](int j, bool p, int w) {
        if (patches[j] < 0) {
            patches[j] = p ? 1 : 0;
            width[j] = w;
        } else {
            patches[j] = (patches[j] && p) ? 1 : 0;
            width[j] = std::max(width[j], w);
        }
    };
    auto through = [&](const Layer& L, bool p, int w, int& w_out) {
        w_out = (w - 1) * L.sw + L.kw;
        return p && L.conv && w_out <= L.in.W;
    };
    for (int m = st; m >= 1; --m) {
        const bool p = patches[m] == 1;
        int w2;
        const bool p2 = through(layers_[m - 1], p, width[m], w2);
        join(m - 1, p2, w2);
        for (const SkipEdge& sk : skips_[m]) {
            if (sk.L) {
                const bool p3 = through(*sk.L, p, width[m], w2);
                join(sk.src, p3, w2);
            } else {
                join(sk.src, p, width[m]);
            }
        }
    }
    return patches[0] == 1 ? CONC_PATCHES : CONC_DENSE;
}

std::string Model::describe() const {
    std::string j = "{\"levels\": [";
    for (int m = 0; m <= K_; ++m) {
        const MapShape& ms = map(m);
        if (m) j += ", ";
        j += "{\"level\": " + std::to_string(m);
        j += ", \"node\": " + std::to_string(m == 0 ? -1 : (m < K_ ? preact_node_ids_[m - 1] : -2));
        j += ", \"map\": [" + std::to_string(ms.C) + ", " + std::to_string(ms.H) + ", " + std::to_string(ms.W) + "]";
        j += std::string(", \"act\": \"") + (act_[m] == ACT_RELU ? "relu" : act_[m] == ACT_SIGMOID ? "sigmoid" : "") + "\"";
        if (m) {
            const Layer& L = layers_[m - 1];
            j += std::string(", \"edge\": \"") + (L.convt ? "convt" : L.conv ? "conv" : "linear") + "\"";
            j += ", \"skips\": [";
            for (size_t e = 0; e < skips_[m].size(); ++e) {
                if (e) j += ", ";
                j += "{\"src\": " + std::to_string(skips_[m][e].src) + ", \"conv\": " +
                     (skips_[m][e].L ? "true" : "false") + "}";
            }
            j += "]";
        }
        j += "}";
    }
    j += "], \"starts\": [";
    for (int st = 2; st <= K_; ++st) {
        if (st > 2) j += ", ";
        j += "{\"level\": " + std::to_string(st) + ", \"form\": \"" +
             (start_form(st) == CONC_PATCHES ? "patches" : "dense") + "\", \"windows\": [";
        for (int m = 0; m <= st; ++m) {
            const WinGeo& g = geo_[st][m];
            if (m) j += ", ";
            j += "[" + std::to_string(g.wh) + ", " + std::to_string(g.ww) + ", " + std::to_string(g.mul_y) + ", " +
                 std::to_string(g.off_y) + ", " + std::to_string(g.full) + "]";
        }
        j += "]}";
    }
    return j + "]}";
}

SkipStep Model::skip_step(int st, int m, int e) const {
    const SkipEdge& sk = skips_[m][e];
    const WinGeo& gi = geo_[st][m];
    const WinGeo& go = geo_[st][sk.src];
    SkipStep k;
    k.gi = gi;
    k.go = go;
    k.Co = map(m).C;
    k.Ci = map(sk.src).C;
    if (sk.L) {
        const Layer& L = *sk.L;
        k.kh = L.kh;
        k.kw = L.kw;
        k.sh = L.sh;
        k.sw = L.sw;
        k.Wk = L.Wt;
        k.Wc = L.W;
        // q s + k = v + c with c = off_j - off_i s + p (offsets 0 on whole maps).
        k.cy = go.off_y - gi.off_y * L.sh + L.ph;
        k.cx = go.off_x - gi.off_x * L.sw + L.pw;
    } else {
        k.cy = go.off_y - gi.off_y;
        k.cx = go.off_x - gi.off_x;
    }
    return k;
}

bool Model::skip_source(int st, int j, bool with_start) const {
    for (int m = j + 2; m <= (with_start ? st : st - 1); ++m)
        for (const SkipEdge& sk : skips_[m])
            if (sk.src == j) return true;
    return false;
}

Model::~Model() {
    if (!on_device_) return;
    cudaSetDevice(device_);
    for (auto e : ev_pool_) cudaEventDestroy(e);
    cache_.release();
    weights_.release();
}

std::string Model::key(const char* what, int a, int b) const {
    std::string k(what);
    k += "/" + std::to_string(a);
    if (b >= 0) k += "/" + std::to_string(b);
    return k;
}

size_t Model::bytes_per_box(bool alpha, int nspec) const {
    // Worst case (every neuron unstable).  Persistent per start: signs, row
    // maps and partial sums, plus alpha / Adam m, v / best alpha / saved P per
    // level in alpha mode; transient (largest start): two Q, two P, two Pbar
    // and one Qbar buffer, plus the skip sums S_j and kept Pbar_j of the
    // levels that feed skip edges.
    size_t total = 0, transient = 0;
    for (int s = 2; s <= K_; ++s) {
        const size_t rows = 2 * (size_t)(s == K_ ? nspec : width(s));
        size_t per_row = (size_t)rowlen(s, 0) + 96;
        size_t maxrow = 0, skiprow = 0;
        for (int m = 0; m < s; ++m) {
            maxrow = std::max(maxrow, (size_t)rowlen(s, m));
            if (alpha && m >= 1) per_row += (size_t)rowlen(s, m) * 4 * ((warm_keep_ || warm_pending_) ? 6 : 5);
            if (m >= 1 && skip_source(s, m, true)) skiprow += (size_t)rowlen(s, m) * 4 * 2;
        }
        total += rows * per_row;
        transient = std::max(transient, rows * (maxrow * 4 * 7 + skiprow));
    }
    for (int m = 0; m <= K_; ++m) total += (size_t)width(m) * 4 * 16;
    // Warm start: per-start relaxation parameters and creation sets.
    if (alpha && (warm_keep_ || warm_pending_))
        for (int m = 1; m < K_; ++m) total += (size_t)width(m) * 16 * (K_ - m);
    return total + transient + (size_t)nspec * 64;
}

// ------------------------------------------------------------ row maps
void Model::build_rows(int B, int nspec, cudaStream_t s) {
    starts_.assign(K_ + 1, StartPlan{});
    std::vector<int> totals(K_ + 1, 0);
    for (int st = 2; st < K_; ++st) {
        StartPlan& sp = starts_[st];
        sp.s = st;
        int* counts = cache_.as<int>(key("counts", st), B);
        sp.box_off = cache_.as<int>(key("boxoff", st), B + 1);
        launch_count_unstable(cache_.as<float>(key("ibp_l", st), (size_t)B * width(st)),
                              cache_.as<float>(key("ibp_u", st), (size_t)B * width(st)), B, width(st),
                              counts, s);
        launch_scan_counts(counts, B, sp.box_off, s);
    }
    // One synchronisation for all row totals.
    std::vector<int> host(K_ + 1, 0);
    for (int st = 2; st < K_; ++st)
        LB_CUDA(cudaMemcpyAsync(&host[st], starts_[st].box_off + B, sizeof(int), cudaMemcpyDeviceToHost, s));
    LB_CUDA(cudaStreamSynchronize(s));
    for (int st = 2; st < K_; ++st) {
        StartPlan& sp = starts_[st];
        const int R = host[st];
        sp.row_box = cache_.as<int>(key("rowbox", st), std::max(R, 1));
        sp.row_id = cache_.as<int>(key("rowid", st), std::max(R, 1));
        const float* il = cache_.as<float>(key("ibp_l", st), (size_t)B * width(st));
        const float* iu = cache_.as<float>(key("ibp_u", st), (size_t)B * width(st));
        if (map(st).spatial)
            // Rows in Luna's (CHW) neuron order; row_id is the HWC index.
            launch_fill_rows_chw(il, iu, B, map(st).C, map(st).H, map(st).W, sp.box_off, sp.row_box,
                                 sp.row_id, s);
        else
            launch_fill_rows(il, iu, B, width(st), sp.box_off, sp.row_box, sp.row_id, s);
        sp.rows = RowMap{sp.row_box, sp.row_id, sp.box_off, R};
        sp.geo = geo_[st];
        sp.form = start_form(st);
    }
    StartPlan& out = starts_[K_];
    out.s = K_;
    const int R = B * nspec;
    out.row_box = cache_.as<int>(key("rowbox", K_), std::max(R, 1));
    out.row_id = cache_.as<int>(key("rowid", K_), std::max(R, 1));
    out.box_off = cache_.as<int>(key("boxoff", K_), B + 1);
    launch_fill_spec_rows(B, nspec, out.row_box, out.row_id, out.box_off, s);
    out.rows = RowMap{out.row_box, out.row_id, out.box_off, R};
    out.geo = geo_[K_];
    out.form = CONC_DENSE;
}

// ------------------------------------------------------------ relaxation
void Model::relu_params(int m, int B, bool alpha_mode, bool create, cudaStream_t s) {
    const int n = width(m);
    const size_t bn = (size_t)B * n;
    if (act_[m] == ACT_SIGMOID) {
        // No alpha for a Sigmoid (Luna cannot create one: its 8-slot init
        // throws, AlphaCROWNAnalysis.cpp:264-272); the CROWN relaxation stays.
        if (create) LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("init", m), bn), 0, bn * 4, s));
        launch_sigmoid_params(cache_.as<float>(key("cur_l", m), bn), cache_.as<float>(key("cur_u", m), bn), B, n,
                              cache_.as<float>(key("rp_s", m), bn), cache_.as<float>(key("rp_bl", m), bn),
                              cache_.as<float>(key("rp_k", m), bn), cache_.as<float>(key("rp_b", m), bn),
                              cache_.as<uint8_t>(key("rp_f", m), bn), s);
        return;
    }
    launch_relu_params(cache_.as<float>(key("cur_l", m), bn), cache_.as<float>(key("cur_u", m), bn), B,
                       n, alpha_mode, create, cache_.as<uint8_t>(key("aset", m), bn),
                       cache_.as<float>(key("init", m), bn), cache_.as<int>(key("hasaset", m), B),
                       cache_.as<float>(key("rp_s", m), bn), cache_.as<float>(key("rp_k", m), bn),
                       cache_.as<float>(key("rp_b", m), bn), cache_.as<uint8_t>(key("rp_f", m), bn), s);
}

ReluParams Model::rview(int m, int B, int n, int st) {
    ReluParams rp;
    const size_t bn = (size_t)B * n;
    if (warm_on_ && alpha_ && st > m) {
        rp.slope_lo = cache_.as<float>(key("wrp_s", m, st), bn);
        rp.k_up = cache_.as<float>(key("wrp_k", m, st), bn);
        rp.b_up = cache_.as<float>(key("wrp_b", m, st), bn);
        rp.flags = cache_.as<uint8_t>(key("wrp_f", m, st), bn);
        rp.n = n;
        return rp;
    }
    rp.slope_lo = cache_.as<float>(key("rp_s", m), bn);
    rp.k_up = cache_.as<float>(key("rp_k", m), bn);
    rp.b_up = cache_.as<float>(key("rp_b", m), bn);
    rp.flags = cache_.as<uint8_t>(key("rp_f", m), bn);
    if (act_[m] == ACT_SIGMOID) rp.b_lo = cache_.as<float>(key("rp_bl", m), bn);
    rp.n = n;
    return rp;
}

// ------------------------------------------------------------ warm start
// A seeded alpha keeps the creation set (unstableIndices) its parent's run
// made it with (AlphaCROWNAnalysis::seedAlphas, AlphaCROWNAnalysis.cpp:971-997),
// so the ReLU relaxation of level m differs per start: each start above m
// reads its own parameters, with every box's creation set (the parent's where
// the box is seeded for that start, its own otherwise).  Only ReLU levels
// reach here (a warm start is refused on networks with a Sigmoid).
void Model::warm_relu_params(int m, int B, bool create, cudaStream_t s) {
    const int n = width(m);
    const size_t bn = (size_t)B * n;
    for (int st = m + 1; st <= K_; ++st) {
        uint8_t* wa = cache_.as<uint8_t>(key("waset", m, st), bn);
        int* wh = cache_.as<int>(key("whas", m, st), B);
        if (create)
            launch_warm_aset(cache_.as<int>(key("wseed", st), B), cache_.as<int>("wparent", B), B, n,
                             cache_.as<uint8_t>(key("w_aset", m, st), (size_t)warm_B_ * n),
                             cache_.as<uint8_t>(key("aset", m), bn), wa, wh, s);
        launch_relu_params(cache_.as<float>(key("cur_l", m), bn), cache_.as<float>(key("cur_u", m), bn), B, n,
                           true, false, wa, cache_.as<float>(key("init", m), bn), wh,
                           cache_.as<float>(key("wrp_s", m, st), bn), cache_.as<float>(key("wrp_k", m, st), bn),
                           cache_.as<float>(key("wrp_b", m, st), bn), cache_.as<uint8_t>(key("wrp_f", m, st), bn), s);
    }
}

// TorchModel::getState after the call (TorchModel.cpp:995-1014): the alphas
// extractAlphas returns (the best ones, which restoreBestAlphas has just made
// current), with the creation sets they were made with, and each start's
// rows per box.
void Model::warm_retain(int B, cudaStream_t s) {
    warm_R_.assign(K_ + 1, 0);
    for (int st = 2; st <= K_; ++st) {
        const StartPlan& sp = starts_[st];
        warm_R_[st] = sp.rows.R;
        LB_CUDA(cudaMemcpyAsync(cache_.as<int>(key("w_boxoff", st), B + 1), sp.box_off, (size_t)(B + 1) * 4,
                                cudaMemcpyDeviceToDevice, s));
        for (int m = 1; m < st; ++m) {
            const size_t cnt = (size_t)2 * sp.rows.R * rowlen(st, m);
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("w_alpha", m, st), cnt),
                                    cache_.as<float>(key("alpha", m, st), cnt), cnt * 4, cudaMemcpyDeviceToDevice, s));
            const size_t bn = (size_t)B * width(m);
            const uint8_t* src = warm_on_ ? cache_.as<uint8_t>(key("waset", m, st), bn)
                                          : cache_.as<uint8_t>(key("aset", m), bn);
            LB_CUDA(cudaMemcpyAsync(cache_.as<uint8_t>(key("w_aset", m, st), bn), src, bn, cudaMemcpyDeviceToDevice,
                                    s));
        }
    }
    warm_B_ = B;
    warm_valid_ = true;
}

void Model::set_warm_parents(const int64_t* parent, int64_t n) {
    if (n < 0 || (n > 0 && !parent)) throw std::invalid_argument("set_warm_parents: bad arguments");
    if (!warm_valid_)
        throw std::invalid_argument(
            "set_warm_parents: no retained state (run an alpha-CROWN call with warm start on first)");
    std::vector<int> p((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        if (parent[i] < -1 || parent[i] >= warm_B_)
            throw std::invalid_argument("set_warm_parents: parent index out of range of the retained boxes");
        p[(size_t)i] = (int)parent[i];
    }
    warm_parent_ = std::move(p);
    warm_pending_ = true;
}

void Model::warm_alpha(int m, int st, int64_t box, float* out, int64_t cap, int64_t* rows, int64_t* cols,
                       uint8_t* aset) {
    if (!warm_valid_) throw std::invalid_argument("warm_alpha: no retained state");
    if (st < 2 || st > K_ || m < 1 || m >= st) throw std::invalid_argument("warm_alpha: bad level or start");
    if (box < 0 || box >= warm_B_) throw std::invalid_argument("warm_alpha: box out of range of the retained boxes");
    const int n = rowlen(st, m), R = warm_R_[st];
    int bo[2] = {0, 0};
    LB_CUDA(cudaSetDevice(device_));
    LB_CUDA(cudaMemcpy(bo, cache_.as<int>(key("w_boxoff", st), warm_B_ + 1) + box, 2 * sizeof(int),
                       cudaMemcpyDeviceToHost));
    const int64_t nr = bo[1] - bo[0];
    *rows = nr;
    *cols = n;
    const float* a = cache_.as<float>(key("w_alpha", m, st), (size_t)2 * R * n);
    if (out && cap >= 2 * nr * n && nr > 0) {
        LB_CUDA(cudaMemcpy(out, a + (size_t)bo[0] * n, (size_t)nr * n * 4, cudaMemcpyDeviceToHost));
        LB_CUDA(cudaMemcpy(out + nr * n, a + ((size_t)R + bo[0]) * n, (size_t)nr * n * 4, cudaMemcpyDeviceToHost));
    }
    if (aset)
        LB_CUDA(cudaMemcpy(aset, cache_.as<uint8_t>(key("w_aset", m, st), (size_t)warm_B_ * width(m)) + box * width(m),
                           (size_t)width(m), cudaMemcpyDeviceToHost));
}

// ------------------------------------------------------------ forward start
// Backward substitution from start sp.s (CROWNAnalysis::backwardFrom) down to
// the input, both sides stacked, ending in the concretisation
// (computeConcreteLowerBound/UpperBound).  Row totals land in "val/s".
void Model::forward_start(StartPlan& sp, int B, int nspec, bool save, bool alpha, cudaStream_t s) {
    if (tc_) {
        forward_start_tc(sp, B, nspec, save, alpha, s);
        return;
    }
    const int st = sp.s;
    const int R = sp.rows.R;
    if (R == 0) return;
    const int M = 2 * R;
    int maxw = 0;
    for (int m = 0; m < st; ++m) maxw = std::max(maxw, rowlen(st, m));
    float* Q[2] = {cache_.as<float>(key("Q", 0), (size_t)M * maxw), cache_.as<float>(key("Q", 1), (size_t)M * maxw)};
    float* bias = cache_.as<float>(key("bias", st), M);
    const int mb = st - 1;  // ReLU directly below the start
    // Conv layers above the first run on tensor cores when their shapes allow.
    auto tc_fwd = [&](int m) { return tcconv_ && m >= 2 && layers_[m - 1].tcf; };
    int slots_total = 0;
    auto tct_back = [&](int m) { return tcconv_ && layers_[m - 1].convt && layers_[m - 1].tct_b; };
    for (int m = mb; m >= 1; --m) {
        if (tct_back(m))
            slots_total += relax_window_chunks(sp.geo[m - 1]);
        else if (layers_[m - 1].convt)
            slots_total += convt_rb_ok(convt_step(m)) ? convt_rb_chunks(convt_step(m)) : conv_chunks(sp.geo[m - 1]);
        else if (!layers_[m - 1].conv)
            slots_total += gemm_tiles_n(width(m - 1));
        else if (m == 1 && first_conv_fast(conv_step(st, 1)))
            slots_total += 1;
        else if (tc_fwd(m))
            slots_total += relax_window_chunks(sp.geo[m - 1]);
        else if (m >= 2 && convT_rb_ok(conv_step(st, m)))
            slots_total += convT_rb_chunks(sp.geo[m - 1]);
        else
            slots_total += conv_chunks(sp.geo[m - 1]);
    }
    float* part = cache_.as<float>(key("part", st), (size_t)slots_total * M);
    auto alpha_buf = [&](int m) {
        return alpha ? cache_.as<float>(key("alpha", m, st), (size_t)M * rowlen(st, m)) : nullptr;
    };
    auto psave_buf = [&](int m) {
        return save ? cache_.as<float>(key("Psave", st, m), (size_t)M * rowlen(st, m)) : nullptr;
    };
    // Residual joins: S_j collects the A that skip edges carry to level j; it
    // joins the main path's A in the step that relaxes level j.
    auto S_buf = [&](int j) { return cache_.as<float>(key("S", j), (size_t)M * rowlen(st, j)); };
    auto addend = [&](int j) { return j >= 1 && skip_source(st, j, true) ? S_buf(j) : nullptr; };
    auto run_skips = [&](int m, const float* Qm) {
        for (size_t e = 0; e < skips_[m].size(); ++e)
            launch_skip_back(skip_step(st, m, (int)e), sp.rows, M, Qm, S_buf(skips_[m][e].src), s);
    };
    for (int j = 1; j < st; ++j)
        if (addend(j)) LB_CUDA(cudaMemsetAsync(S_buf(j), 0, (size_t)M * rowlen(st, j) * 4, s));
    run_skips(st, nullptr);  // the start's own skip edges carry its one-hot rows

    const Layer& Ls = layers_[st - 1];
    if (Ls.conv || Ls.convt) {
        // Conv start: identity patches through the start conv; ConvTranspose
        // start: the one-hot rows through the layer (whole maps).
        ConvStartStep cs;
        cs.rows = sp.rows;
        cs.M = M;
        cs.Wc = Ls.W;
        cs.bW = Ls.convt ? Ls.b : level_bias(st);  // main and skip-conv biases of the start level
        cs.g = sp.geo[mb];
        if (Ls.conv && cs.g.full) {
            // Whole-map rows of a conv start: the weight window sits at the
            // start pixel's receptive field inside the map.
            WinGeo w = cs.g;
            w.full = 0;
            w.wh = Ls.kh;
            w.ww = Ls.kw;
            w.mul_y = Ls.sh;
            w.mul_x = Ls.sw;
            w.off_y = -Ls.ph;
            w.off_x = -Ls.pw;
            w.st_C = Ls.out.C;
            w.st_W = Ls.out.W;
            cs.wg = w;
        }
        cs.rp = rview(mb, B, width(mb), st);
        cs.alpha = alpha_buf(mb);
        cs.b_next = level_bias(mb);
        cs.P_save = psave_buf(mb);
        cs.Q = Q[0];
        cs.bias_acc = bias;
        if (Ls.convt)
            launch_convt_start_step(cs, convt_step(st), s);
        else
            launch_conv_start_step(cs, s);
    } else {
        StartStep ss;
        ss.rows = sp.rows;
        ss.M = M;
        ss.W = Ls.W;
        ss.bW = Ls.b;
        ss.spec_dim = Ls.n_out;
        ss.n = Ls.n_in;
        if (st == K_) {
            ss.C = C_;
            ss.c_per_box = c_per_box_;
            ss.nspec = nspec;
            flops_ += 2.0 * M * (double)Ls.n_in * Ls.n_out;
        }
        ss.rp = rview(mb, B, width(mb), st);
        ss.alpha = alpha_buf(mb);
        ss.b_next = level_bias_n(mb);
        ss.P_save = psave_buf(mb);
        ss.Q = Q[0];
        ss.bias_acc = bias;
        launch_start_step(ss, s);
    }

    int cur = 0, slot = 0;
    for (int m = mb; m >= 1; --m) {
        const Layer& L = layers_[m - 1];
        run_skips(m, Q[cur]);
        if (L.convt) {
            // k > 1 for a transposed conv (checked at model creation).
            const ConvTStep ct = convt_step(m);
            const double fl = 2.0 * M * (double)rowlen(st, m) * ct.Ci * L.kh * L.kw / ((double)L.sh * L.sw);
            flops_ += fl;
            ConvRelaxEpi e;
            e.rows = sp.rows;
            e.g = sp.geo[m - 1];
            e.rp = rview(m - 1, B, width(m - 1), st);
            e.alpha = alpha_buf(m - 1);
            e.b_next = level_bias(m - 1);
            e.P_save = psave_buf(m - 1);
            e.Q = Q[1 - cur];
            prof_begin(s);
            if (tct_back(m)) {
                // Tensor cores: the strided correlation stores raw P (into the
                // saved P when the adjoint needs it), then the relaxation of
                // the level below streams over it.
                TcConvQbar q;
                q.Co = L.in.C;
                q.in_w = L.in.W;
                q.Qbar = e.P_save ? e.P_save : cache_.as<float>("Pconv", (size_t)M * rowlen(st, m - 1));
                launch_tc_conv_qbar(tct_back_plan(m, M, Q[cur]), M, q, s);
                prof_end(s, fl);
                launch_relax_window(q.Qbar, e, M, part + (size_t)slot * M, s);
                slot += relax_window_chunks(sp.geo[m - 1]);
                cur = 1 - cur;
                continue;
            }
            if (convt_rb_ok(ct)) {
                launch_convt_back_relax_rb(Q[cur], ct, M, e, part + (size_t)slot * M, s);
                slot += convt_rb_chunks(ct);
            } else {
                launch_convt_back_relax(Q[cur], ct, M, e, part + (size_t)slot * M, s);
                slot += conv_chunks(sp.geo[m - 1]);
            }
            prof_end(s, fl);
            cur = 1 - cur;
            continue;
        }
        if (L.conv) {
            const ConvStep cs = conv_step(st, m);
            const double fl = 2.0 * M * (double)rowlen(st, m - 1) * cs.Co * L.kh * L.kw /
                              ((double)L.sh * L.sw);
            flops_ += fl;
            prof_begin(s);
            if (m - 1 >= 1) {
                ConvRelaxEpi e;
                e.rows = sp.rows;
                e.g = sp.geo[m - 1];
                e.rp = rview(m - 1, B, width(m - 1), st);
                e.alpha = alpha_buf(m - 1);
                e.b_next = level_bias(m - 1);
                e.P_save = psave_buf(m - 1);
                e.Q = Q[1 - cur];
                e.addend = addend(m - 1);
                if (tc_fwd(m)) {
                    // Raw P from the tensor cores (into the saved P when the
                    // adjoint needs it), then the relaxation streams over it.
                    TcConvFwd f;
                    f.s = L.sh;
                    f.Ci = L.in.C;
                    int nty, ntx;
                    conv_phase(st, m, f.cy, f.cx, f.tlo_y, f.tlo_x, nty, ntx);
                    f.out_h = sp.geo[m - 1].wh;
                    f.out_w = sp.geo[m - 1].ww;
                    f.P = e.P_save ? e.P_save : cache_.as<float>("Pconv", (size_t)M * rowlen(st, m - 1));
                    launch_tc_conv_fwd(tc_fwd_plan(st, m, M, Q[cur]), M, f, s);
                    prof_end(s, fl);
                    launch_relax_window(f.P, e, M, part + (size_t)slot * M, s);
                    slot += relax_window_chunks(sp.geo[m - 1]);
                    cur = 1 - cur;
                    continue;
                }
                if (convT_rb_ok(cs)) {
                    launch_convT_relax_rb(Q[cur], cs, M, e, part + (size_t)slot * M, s);
                    prof_end(s, fl);
                    slot += convT_rb_chunks(sp.geo[m - 1]);
                    cur = 1 - cur;
                    continue;
                }
                launch_convT_relax(Q[cur], cs, M, e, part + (size_t)slot * M, s);
                cur = 1 - cur;
            } else {
                ConvConcEpi e;
                e.rows = sp.rows;
                e.g = sp.geo[0];
                e.form = sp.form;
                e.xl = xl_;
                e.xu = xu_;
                if (save) e.sign = cache_.as<uint8_t>(key("sign", st), (size_t)M * rowlen(st, 0));
                if (first_conv_fast(cs)) {
                    launch_first_convT_conc(Q[cur], cs, M, e, part + (size_t)slot * M, s);
                    prof_end(s, fl);
                    slot += 1;
                    continue;
                }
                launch_convT_conc(Q[cur], cs, M, e, part + (size_t)slot * M, s);
            }
            prof_end(s, fl);
            slot += conv_chunks(sp.geo[m - 1]);
            continue;
        }
        const int N = L.n_in, Kd = L.n_out;
        flops_ += 2.0 * M * (double)N * Kd;
        if (m - 1 >= 1) {
            EpiRelaxFwd e;
            e.rows = sp.rows;
            e.rp = rview(m - 1, B, width(m - 1), st);
            e.alpha = alpha_buf(m - 1);
            e.b_next = level_bias_n(m - 1);
            e.P_save = psave_buf(m - 1);
            e.Q = Q[1 - cur];
            prof_begin(s);
            launch_gemm_relax_fwd(Q[cur], L.W, M, N, Kd, e, part + (size_t)slot * M, s);
            prof_end(s, 2.0 * M * (double)N * Kd);
            cur = 1 - cur;
        } else {
            EpiConcretize e;
            e.rows = sp.rows;
            e.xl = xl_;
            e.xu = xu_;
            if (save) e.sign = cache_.as<uint8_t>(key("sign", st), (size_t)M * N);
            prof_begin(s);
            launch_gemm_concretize(Q[cur], L.W, M, N, Kd, e, part + (size_t)slot * M, s);
            prof_end(s, 2.0 * M * (double)N * Kd);
        }
        slot += gemm_tiles_n(N);
    }
    launch_sum_partials(bias, part, slot, M, cache_.as<float>(key("val", st), M), s);
    rows_ += M;
}

// Tensor-core schedule of the same pass.  A contraction whose N fits one
// column tile forms its A operand in its prologue (the relaxation of the P
// below it, or of the one-hot rows of W for an intermediate start) and the
// step before it stores only the raw P; a contraction with several column
// tiles reads a materialised Q by TMA instead (forming it in the prologue
// would redo the relaxation once per column tile), and the step before it
// relaxes in its epilogue.  Per-row bias sums come from prologues (one slot
// each), relaxing epilogues and the concretisation (one slot per column tile).
void Model::forward_start_tc(StartPlan& sp, int B, int nspec, bool save, bool alpha, cudaStream_t s) {
    const int st = sp.s;
    const int R = sp.rows.R;
    if (R == 0) return;
    const int M = 2 * R;
    const int mb = st - 1;
    int maxw = 0;
    for (int m = 0; m < st; ++m) maxw = std::max(maxw, width(m));
    auto in_prologue = [&](int m) { return tc_tiles_n(width(m - 1), pairs_) == 1; };
    int slots_total = 0;
    for (int m = 1; m <= mb; ++m) slots_total += 1 + tc_tiles_n(width(m - 1), pairs_);
    float* part = cache_.as<float>(key("part", st), (size_t)slots_total * M);
    float* Qbuf[2] = {cache_.as<float>(key("Q", 0), (size_t)M * maxw), cache_.as<float>(key("Q", 1), (size_t)M * maxw)};
    float* Pscr[2] = {nullptr, nullptr};
    if (!save)
        for (int i = 0; i < 2; ++i) Pscr[i] = cache_.as<float>(key("Pfwd", i), (size_t)M * maxw);
    int qcur = 0, pcur = 0, slot = 0;
    float* base = nullptr;
    const float* P_in = nullptr;  // raw P below the next contraction (prologue modes)
    const float* Q_in = nullptr;  // materialised A of the next contraction (TMA mode)
    const Layer& Ls = layers_[st - 1];
    if (st == K_ || !in_prologue(mb)) {
        // Start step: P = C . W_K (output start) or the one-hot rows of W_s,
        // relaxed here when the first contraction reads a materialised Q.
        StartStep ss;
        ss.rows = sp.rows;
        ss.M = M;
        ss.W = Ls.W;
        ss.bW = Ls.b;
        ss.spec_dim = Ls.n_out;
        ss.n = Ls.n_in;
        if (st == K_) {
            ss.C = C_;
            ss.c_per_box = c_per_box_;
            ss.nspec = nspec;
            ss.P_save = cache_.as<float>(key("Psave", st, mb), (size_t)M * width(mb));
            flops_ += 2.0 * M * (double)Ls.n_in * Ls.n_out;
        }
        if (!in_prologue(mb)) {
            ss.rp = rview(mb, B, width(mb), st);
            if (alpha) ss.alpha = cache_.as<float>(key("alpha", mb, st), (size_t)M * width(mb));
            ss.b_next = layers_[mb - 1].b;
            ss.Q = Qbuf[qcur];
            Q_in = Qbuf[qcur];
            qcur ^= 1;
        } else {
            P_in = ss.P_save;
        }
        base = cache_.as<float>(key("bias", st), M);
        ss.bias_acc = base;
        launch_start_step(ss, s);
    }
    for (int m = mb; m >= 1; --m) {
        const Layer& L = layers_[m - 1];
        const int N = L.n_in, Kd = L.n_out;
        TcPrologue pro;
        if (in_prologue(m)) {
            pro.rows = sp.rows;
            pro.rp = rview(m, B, Kd, st);
            if (alpha) pro.alpha = cache_.as<float>(key("alpha", m, st), (size_t)M * Kd);
            pro.b_lin = L.b;
            if (m == mb && st != K_) {
                pro.gather_W = Ls.W;
                pro.gather_b = Ls.b;
            } else {
                pro.P = P_in;
            }
            pro.bias_part = part + (size_t)slot * M;
            ++slot;
        }
        const float* A = in_prologue(m) ? nullptr : Q_in;
        flops_ += 2.0 * M * (double)N * Kd;
        prof_begin(s);
        if (m == 1) {
            EpiConcretize e;
            e.rows = sp.rows;
            e.xl = xl_;
            e.xu = xu_;
            if (save) e.sign = cache_.as<uint8_t>(key("sign", st), (size_t)M * N);
            launch_tc_forward(A, pro, L.Wt_hi, L.Wt_lo, M, N, Kd, nullptr, nullptr, &e, part + (size_t)slot * M, pairs_, split_fwd_, s);
            slot += tc_tiles_n(N, pairs_);
        } else if (in_prologue(m - 1)) {
            float* P_out = save ? cache_.as<float>(key("Psave", st, m - 1), (size_t)M * N) : Pscr[pcur];
            pcur ^= 1;
            launch_tc_forward(A, pro, L.Wt_hi, L.Wt_lo, M, N, Kd, P_out, nullptr, nullptr, nullptr, pairs_, split_fwd_, s);
            P_in = P_out;
        } else {
            EpiRelaxFwd e;
            e.rows = sp.rows;
            e.rp = rview(m - 1, B, N, st);
            if (alpha) e.alpha = cache_.as<float>(key("alpha", m - 1, st), (size_t)M * N);
            e.b_next = layers_[m - 2].b;
            if (save) e.P_save = cache_.as<float>(key("Psave", st, m - 1), (size_t)M * N);
            e.Q = Qbuf[qcur];
            launch_tc_forward(A, pro, L.Wt_hi, L.Wt_lo, M, N, Kd, nullptr, &e, nullptr, part + (size_t)slot * M, pairs_, split_fwd_, s);
            slot += tc_tiles_n(N, pairs_);
            Q_in = Qbuf[qcur];
            qcur ^= 1;
        }
        prof_end(s, 2.0 * M * (double)N * Kd);
    }
    launch_sum_partials(base, part, slot, M, cache_.as<float>(key("val", st), M), s);
    rows_ += M;
}

// ------------------------------------------------------------ adjoint start
// Reverse sweep of forward_start for M stacked rows with seeds g (d loss /
// d bound of each row).  Produces d loss / d alpha(m, s) for every ReLU m
// below the start and accumulates d loss / d (k_up, b_up) of those ReLUs.
void Model::adjoint_start(StartPlan& sp, int B, const float* g, int M, cudaStream_t s) {
    const int st = sp.s;
    const int R = sp.rows.R;
    if (R == 0 || M == 0) return;
    // Conv layers above the first take their adjoint on tensor cores when
    // their shapes allow; the Pbar below such a layer is stored phase-split.
    auto tc_adj = [&](int m) { return tcconv_ && m >= 2 && m <= st - 1 && layers_[m - 1].tca; };
    int64_t maxw = 0;
    for (int m = 0; m < st; ++m) {
        maxw = std::max<int64_t>(maxw, rowlen(st, m));
        if (m >= 1 && tc_adj(m + 1)) maxw = std::max<int64_t>(maxw, phase_split(st, m + 1).row_stride);
    }
    float* Pb[2] = {cache_.as<float>(key("Pbar", 0), (size_t)M * maxw),
                    cache_.as<float>(key("Pbar", 1), (size_t)M * maxw)};
    const int n0 = width(0);
    const uint8_t* sign = cache_.as<uint8_t>(key("sign", st), (size_t)2 * R * rowlen(st, 0));
    // On the tensor-core path the first contraction generates d loss / d A at
    // the input from the signs itself; the SIMT path materialises it.
    const bool tc_adj_gemm = tc_ && !simt_adjoint_;  // tensor-core adjoint contractions
    const bool seed_in_kernel = tc_adj_gemm;
    // A small first conv generates the input seed inside its adjoint kernel.
    const bool first_fast = layers_[0].conv && first_conv_fast(conv_step(st, 1));
    if (layers_[0].conv) {
        if (!first_fast) launch_win_input_seed(sp.rows, M, sp.geo[0], sp.form, sign, g, xl_, xu_, Pb[0], s);
    } else if (!seed_in_kernel) {
        launch_adj_input_seed(sp.rows, M, sign, g, xl_, xu_, n0, Pb[0], s);
    }
    // Pbar of a skip source stays in its own buffer until the skip's target
    // level takes its adjoint.
    auto ps_of = [&](int j) { return tc_adj(j + 1) ? phase_split(st, j + 1) : PhaseSplit{}; };
    auto PbS_buf = [&](int j) {
        const int64_t w = std::max<int64_t>(rowlen(st, j), tc_adj(j + 1) ? phase_split(st, j + 1).row_stride : 0);
        return cache_.as<float>(key("PbS", j), (size_t)M * w);
    };
    float* pin = Pb[0];  // Pbar of the level below the current one
    for (int m = 1; m <= st - 1; ++m) {
        const Layer& L = layers_[m - 1];
        const int N = L.n_out, Kd = L.n_in;
        const size_t rl = (size_t)rowlen(st, m);
        float* pout = nullptr;
        if (m < st - 1) pout = skip_source(st, m, false) ? PbS_buf(m) : (pin == Pb[0] ? Pb[1] : Pb[0]);
        auto add_skip_adjoints = [&](float* Qbar) {
            for (size_t k = 0; k < skips_[m].size(); ++k) {
                const int j = skips_[m][k].src;
                launch_skip_adj(skip_step(st, m, (int)k), sp.rows, M, PbS_buf(j), ps_of(j), Qbar, s);
            }
        };
        EpiRelaxAdj e;
        e.rows = sp.rows;
        e.rp = rview(m, B, N, st);
        e.gseed = g;
        e.b_lin = L.b;
        if (tc_ && m == st - 1 && st != K_)
            e.gather_W = layers_[st - 1].W;  // P of the ReLU below a one-hot start
        else
            e.P_saved = cache_.as<float>(key("Psave", st, m), (size_t)2 * R * rl);
        e.alpha = cache_.as<float>(key("alpha", m, st), (size_t)2 * R * rl);
        e.Pbar = pout;
        if (e.Pbar && tc_adj(m + 1)) {
            e.ps = phase_split(st, m + 1);
            LB_CUDA(cudaMemsetAsync(e.Pbar, 0, (size_t)M * e.ps.row_stride * 4, s));
        }
        // Projected Adam fused into the relaxation adjoint (torch::optim::Adam + clip).
        e.adam_m = cache_.as<float>(key("am", m, st), (size_t)2 * R * rl);
        e.adam_v = cache_.as<float>(key("av", m, st), (size_t)2 * R * rl);
        e.active = adam_active_;
        e.adam_step = adam_step_;
        e.adam_bc2_sqrt = adam_bc2_sqrt_;
        e.B = B;
        e.kbar = cache_.as<float>(key("kbar", m), (size_t)B * N);
        e.bbar = cache_.as<float>(key("bbar", m), (size_t)B * N);
        if (L.convt) {
            const ConvTStep ct = convt_step(m);
            const double fl = 2.0 * M * (double)rl * ct.Ci * L.kh * L.kw / ((double)L.sh * L.sw);
            flops_ += fl;
            float* Qbar = cache_.as<float>("Qbar", (size_t)M * rl);
            prof_begin(s);
            if (tcconv_ && L.tct_a) {
                // Tensor cores: the transposed conv of Pbar, phases stacked in M.
                TcConvFwd f;
                f.s = L.sh;
                f.Ci = L.out.C;
                f.cy = L.ph;
                f.cx = L.pw;
                f.tlo_y = L.ph / L.sh;
                f.tlo_x = L.pw / L.sw;
                f.out_h = L.out.H;
                f.out_w = L.out.W;
                f.P = Qbar;
                launch_tc_conv_fwd(tct_adj_plan(m, M, pin), M, f, s);
            } else if (convt_adj_rb_ok(ct)) {
                launch_convt_adj_qbar_rb(pin, ct, M, Qbar, s);
            } else {
                launch_convt_adj_qbar(pin, ct, M, Qbar, s);
            }
            prof_end(s, fl);
            launch_relax_adjoint(e, Qbar, M, N, s);
            pin = pout;
            continue;
        }
        if (L.conv) {
            const ConvStep cs = conv_step(st, m);
            const double fl = 2.0 * M * (double)rowlen(st, m - 1) * cs.Co * L.kh * L.kw /
                              ((double)L.sh * L.sw);
            flops_ += fl;
            float* Qbar = cache_.as<float>("Qbar", (size_t)M * rl);
            prof_begin(s);
            if (m == 1 && first_fast) {
                launch_first_conv_adj(sp.rows, M, sp.geo[0], sp.form, sign, g, xl_, xu_, cs, L.b, Qbar, s);
            } else if (tc_adj(m)) {
                TcConvQbar q;
                q.Co = L.out.C;
                q.in_w = sp.geo[m].ww;
                q.gseed = g;
                q.b = level_bias(m);
                q.Qbar = Qbar;
                launch_tc_conv_qbar(tc_adj_plan(st, m, M, pin), M, q, s);
            } else if (conv_adj_rb_ok(cs)) {
                launch_conv_adj_qbar_rb(pin, cs, M, g, level_bias(m), Qbar, s);
            } else {
                launch_conv_adj_qbar(pin, cs, M, g, level_bias(m), Qbar, s);
            }
            prof_end(s, fl);
            add_skip_adjoints(Qbar);
            if (sp.geo[m].full) {
                launch_relax_adjoint(e, Qbar, M, N, s);
            } else {
                const std::string kk = key("kbar_d", m), bk = key("bbar_d", m);
                const bool fresh = cache_.capacity(kk) < (size_t)B * N * 8;
                e.kbar_d = cache_.as<double>(kk, (size_t)B * N);
                e.bbar_d = cache_.as<double>(bk, (size_t)B * N);
                if (fresh) {
                    LB_CUDA(cudaMemsetAsync(e.kbar_d, 0, (size_t)B * N * 8, s));
                    LB_CUDA(cudaMemsetAsync(e.bbar_d, 0, (size_t)B * N * 8, s));
                }
                launch_relax_adjoint_win(e, sp.geo[m], Qbar, M, s);
                launch_fold_double(e.kbar_d, e.bbar_d, e.kbar, e.bbar, (int64_t)B * N, s);
            }
            pin = pout;
            continue;
        }
        flops_ += 2.0 * M * (double)N * Kd;
        if (tc_adj_gemm) {
            // Tensor cores: the contraction stores Qbar only (compute-bound);
            // the relaxation adjoint + Adam stream through a separate kernel.
            EpiStoreQbar q;
            q.gseed = g;
            q.b_lin = L.b;
            q.Qbar = cache_.as<float>("Qbar", (size_t)M * N);
            q.rows = sp.rows;
            if (m == 1 && seed_in_kernel) {
                q.seed_sign = sign;
                q.seed_xl = xl_;
                q.seed_xu = xu_;
            }
            prof_begin(s);
            launch_tc_store_qbar(pin, L.W_hi, L.W_lo, M, N, Kd, q, pairs_, split_adj_, s);
            prof_end(s, 2.0 * M * (double)N * Kd);
            launch_relax_adjoint(e, q.Qbar, M, N, s);
        } else {
            const size_t nslot = (size_t)relax_grad_slots(M, B, 8) * N;
            e.kslot = cache_.as<float>("kslot", nslot);
            e.bslot = cache_.as<float>("bslot", nslot);
            if (e.rp.b_lo) {
                e.sslot = cache_.as<float>("sslot", nslot);
                e.blslot = cache_.as<float>("blslot", nslot);
            }
            prof_begin(s);
            launch_gemm_relax_adj(pin, L.Wt, M, N, Kd, e, nullptr, s);
            prof_end(s, 2.0 * M * (double)N * Kd);
            launch_reduce_relax_grad(sp.rows, M, B, N, 8, e.kslot, e.bslot, e.kbar, e.bbar, s);
            if (e.rp.b_lo)
                launch_reduce_relax_grad(sp.rows, M, B, N, 8, e.sslot, e.blslot,
                                         cache_.as<float>(key("sbar", m), (size_t)B * N),
                                         cache_.as<float>(key("blbar", m), (size_t)B * N), s);
        }
        pin = pout;
    }
    rows_ += M;
}

// ------------------------------------------------------------ one pass
void Model::run_pass(Pass pass, int B, int nspec, cudaStream_t s) {
    const bool alpha = pass != Pass::CROWN;
    const bool create = pass == Pass::ALPHA_FIRST;
    const bool save = pass == Pass::ALPHA_FIRST || pass == Pass::ALPHA_ITER || pass == Pass::ALPHA_RESTART;
    if (pass == Pass::ALPHA_FINAL) {
        // Intermediate bounds are the best ones (restoreBestIntermediateBounds)
        // and are not recomputed (computeIntermediateBoundsLazy sees node bounds).
        for (int m = 1; m < K_; ++m) {
            const size_t bn = (size_t)B * width(m) * 4;
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("cur_l", m), bn / 4), cache_.as<float>(key("best_l", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("cur_u", m), bn / 4), cache_.as<float>(key("best_u", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
            relu_params(m, B, true, false, s);
            if (warm_on_) warm_relu_params(m, B, false, s);
        }
    } else {
        for (int m = 1; m < K_; ++m) {
            const size_t bn = (size_t)B * width(m);
            float* cl = cache_.as<float>(key("cur_l", m), bn);
            float* cu = cache_.as<float>(key("cur_u", m), bn);
            LB_CUDA(cudaMemcpyAsync(cl, cache_.as<float>(key("ibp_l", m), bn), bn * 4, cudaMemcpyDeviceToDevice, s));
            LB_CUDA(cudaMemcpyAsync(cu, cache_.as<float>(key("ibp_u", m), bn), bn * 4, cudaMemcpyDeviceToDevice, s));
            if (m >= 2) {
                StartPlan& sp = starts_[m];
                if (create)
                    for (int mm = 1; mm < m; ++mm) init_alpha(sp, mm, B, s);
                forward_start(sp, B, nspec, save, alpha, s);
                const bool ste = pass == Pass::ALPHA_ITER && opt_.stabilize_intermediate_bounds;
                launch_scatter_start(sp.rows, cache_.as<float>(key("val", m), (size_t)2 * sp.rows.R),
                                     ste ? cache_.as<float>(key("best_l", m), bn) : nullptr,
                                     ste ? cache_.as<float>(key("best_u", m), bn) : nullptr, width(m), cl, cu, s);
            }
            relu_params(m, B, alpha, create, s);
            if (warm_on_ && alpha) warm_relu_params(m, B, create, s);
        }
    }
    StartPlan& out = starts_[K_];
    if (create)
        for (int mm = 1; mm < K_; ++mm) init_alpha(out, mm, B, s);
    forward_start(out, B, nspec, save, alpha, s);
}

// alpha(m, start) = the CROWN lower slope of ReLU m at creation
// (AlphaCROWNAnalysis::ensureAlphaFor, AlphaCROWNAnalysis.cpp:233-297).
void Model::init_alpha(StartPlan& sp, int m, int B, cudaStream_t s) {
    const float* init = cache_.as<float>(key("init", m), (size_t)B * width(m));
    float* a = cache_.as<float>(key("alpha", m, sp.s), (size_t)2 * sp.rows.R * rowlen(sp.s, m));
    if (sp.geo[m].full)
        launch_alpha_init(sp.rows, init, width(m), a, s);
    else
        launch_alpha_init_win(sp.rows, sp.geo[m], init, width(m), a, s);
    // Warm start: a seeded box takes its parent's alpha rows instead
    // (ensureAlphaFor reuses a seeded alpha whose specification count matches,
    // row by row in order).
    if (warm_on_)
        launch_warm_alpha(sp.rows, cache_.as<int>(key("wseed", sp.s), B), cache_.as<int>("wparent", B),
                          cache_.as<int>(key("w_boxoff", sp.s), warm_B_ + 1), warm_R_[sp.s], rowlen(sp.s, m),
                          cache_.as<float>(key("w_alpha", m, sp.s), (size_t)2 * warm_R_[sp.s] * rowlen(sp.s, m)), a,
                          s);
}

// ------------------------------------------------------------ one chunk
void Model::run_chunk(int method, const float* xl, const float* xu, int B, const float* C,
                      int c_per_box, int nspec, bool upper, float* lb, float* ub, cudaStream_t s) {
    if (in_tf_) {
        // A Sub on the input: the box of x - c (or c - x), in Luna's order,
        // as BoundedSubNode's interval forward computes it.
        float* tl = cache_.as<float>("x_sub_l", (size_t)B * width(0));
        float* tu = cache_.as<float>("x_sub_u", (size_t)B * width(0));
        launch_input_sub(in_const_, in_neg_, xl, xu, tl, tu, B, width(0), s);
        xl = tl;
        xu = tu;
    }
    if (map(0).spatial) {
        // Input boxes arrive in Luna's CHW order; the engine works in HWC.
        const MapShape& m0 = map(0);
        float* pl = cache_.as<float>("x_hwc_l", (size_t)B * m0.n());
        float* pu = cache_.as<float>("x_hwc_u", (size_t)B * m0.n());
        launch_chw_to_hwc(xl, pl, B, m0.C, m0.H, m0.W, s);
        launch_chw_to_hwc(xu, pu, B, m0.C, m0.H, m0.W, s);
        xl = pl;
        xu = pu;
    }
    xl_ = xl;
    xu_ = xu;
    C_ = C;
    tc_ = tc_eligible();
    c_per_box_ = c_per_box;
    const int nout = width(K_);
    // IBP (CROWNAnalysis::computeIBPBounds): pure interval bounds of every
    // affine layer (the ReLU IBP is the clamp applied to each layer's input).
    for (int k = 1; k <= K_; ++k) {
        const size_t bn = (size_t)B * width(k);
        const float* il = k == 1 ? xl : cache_.as<float>(key("ibp_l", k - 1), (size_t)B * width(k - 1));
        const float* iu = k == 1 ? xu : cache_.as<float>(key("ibp_u", k - 1), (size_t)B * width(k - 1));
        bool relu_in = k > 1;
        if (act_[k - 1] == ACT_SIGMOID) {
            // The Sigmoid node's IBP: [sigmoid(l), sigmoid(u)].
            const size_t bp = (size_t)B * width(k - 1);
            float* sl = cache_.as<float>("ibp_sig_l", bp);
            float* su = cache_.as<float>("ibp_sig_u", bp);
            launch_sigmoid_bounds(il, iu, sl, su, (int64_t)bp, s);
            il = sl;
            iu = su;
            relu_in = false;
        }
        const Layer& L = layers_[k - 1];
        float* ol = cache_.as<float>(key("ibp_l", k), bn);
        float* ou = cache_.as<float>(key("ibp_u", k), bn);
        if (L.convt)
            launch_ibp_convt(convt_step(k), L.b, il, iu, ol, ou, B, relu_in, s);
        else if (L.conv)
            launch_ibp_conv(L.W, L.b, il, iu, ol, ou, B, L.in.C, L.in.H, L.in.W, L.out.C, L.out.H, L.out.W, L.kh,
                            L.kw, L.sh, L.sw, L.ph, L.pw, relu_in, s);
        else
            launch_ibp_linear(L.W, L.b, il, iu, ol, ou, B, width(k - 1), width(k), relu_in, s);
        // Add: the interval sum with every skip edge's bounds.
        for (const SkipEdge& sk : skips_[k]) {
            const float* sl = cache_.as<float>(key("ibp_l", sk.src), (size_t)B * width(sk.src));
            const float* su = cache_.as<float>(key("ibp_u", sk.src), (size_t)B * width(sk.src));
            if (!sk.L) {
                launch_add_bounds(ol, ou, sl, su, (int64_t)bn, true, s);
                continue;
            }
            const Layer& P = *sk.L;
            float* tl = cache_.as<float>("ibp_skip_l", bn);
            float* tu = cache_.as<float>("ibp_skip_u", bn);
            launch_ibp_conv(P.W, P.b, sl, su, tl, tu, B, P.in.C, P.in.H, P.in.W, P.out.C, P.out.H, P.out.W, P.kh, P.kw,
                            P.sh, P.sw, P.ph, P.pw, true, s);
            launch_add_bounds(ol, ou, tl, tu, (int64_t)bn, false, s);
        }
    }
    if (method == LB200_METHOD_IBP) {
        launch_ibp_spec(C, c_per_box, cache_.as<float>(key("ibp_l", K_), (size_t)B * nout),
                        cache_.as<float>(key("ibp_u", K_), (size_t)B * nout), B, nspec, nout, lb, ub, s);
        return;
    }
    build_rows(B, nspec, s);
    if (warm_on_)
        for (int st = 2; st <= K_; ++st)
            launch_warm_seed(starts_[st].box_off, cache_.as<int>(key("w_boxoff", st), warm_B_ + 1),
                             cache_.as<int>("wparent", B), B, cache_.as<int>(key("wseed", st), B), s);
    StartPlan& out = starts_[K_];
    float* val_out = nullptr;
    if (method == LB200_METHOD_CROWN) {
        alpha_ = false;
        run_pass(Pass::CROWN, B, nspec, s);
        val_out = cache_.as<float>(key("val", K_), (size_t)2 * out.rows.R);
        launch_scatter_output(out.rows, val_out, nspec, true, lb, ub, s);
        return;
    }
    // TorchModel::compute_bounds (TorchModel.cpp:683-684): a side is optimised
    // when it is computed and its OPTIMIZE_* flag is set.
    const bool opt_upper = upper && opt_.optimize_upper;
    const bool opt_lower = opt_.optimize_lower != 0;
    if (!opt_lower && !opt_upper) {
        // runAlphaCROWN with no side to optimise delegates to runCROWN (:853-857);
        // its pre-activation bounds are the ones reported.
        alpha_ = false;
        run_pass(Pass::CROWN, B, nspec, s);
        for (int m = 1; m < K_; ++m) {
            const size_t bn = (size_t)B * width(m) * 4;
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_l", m), bn / 4), cache_.as<float>(key("cur_l", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_u", m), bn / 4), cache_.as<float>(key("cur_u", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
        }
        launch_scatter_output(out.rows, cache_.as<float>(key("val", K_), (size_t)2 * out.rows.R), nspec, upper, lb, ub,
                              s);
        return;
    }
    BoxControl bc;
    bc.active = cache_.as<int>("ctl_active", B);
    int* active0 = cache_.as<int>("ctl_active0", B);
    int* done = nullptr;
    float* crown_lb = nullptr;
    float* crown_ub = nullptr;
    if (thr_ && opt_.stop_crown_on_verified) {
        // --- TorchModel::runAlphaCROWN early stop (TorchModel.cpp:816-834):
        // the CROWN initialisation pass (AlphaCROWNAnalysis.cpp:118-129, a
        // plain CROWN pass) bounds every box; a box it verifies returns those
        // bounds and takes no part in the optimisation.
        alpha_ = false;
        run_pass(Pass::CROWN, B, nspec, s);
        crown_lb = cache_.as<float>("crown_lb", (size_t)B * nspec);
        crown_ub = cache_.as<float>("crown_ub", (size_t)B * nspec);
        launch_scatter_output(out.rows, cache_.as<float>(key("val", K_), (size_t)2 * out.rows.R), nspec, true,
                              crown_lb, crown_ub, s);
        done = cache_.as<int>("ctl_done", B);
        int* n_done = cache_.as<int>("ctl_ndone", 1);
        LB_CUDA(cudaMemsetAsync(n_done, 0, sizeof(int), s));
        launch_crown_verified(crown_lb, thr_, branch_, n_branches_, B, nspec, done, bc.active, n_done, s);
        int h_done = 0;
        LB_CUDA(cudaMemcpyAsync(&h_done, n_done, sizeof(int), cudaMemcpyDeviceToHost, s));
        LB_CUDA(cudaStreamSynchronize(s));
        if (h_done == B) {
            // Every box verified: the intermediate bounds are the CROWN pass's.
            for (int m = 1; m < K_; ++m) {
                const size_t bn = (size_t)B * width(m) * 4;
                LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_l", m), bn / 4),
                                        cache_.as<float>(key("cur_l", m), bn / 4), bn, cudaMemcpyDeviceToDevice, s));
                LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_u", m), bn / 4),
                                        cache_.as<float>(key("cur_u", m), bn / 4), bn, cudaMemcpyDeviceToDevice, s));
            }
            LB_CUDA(cudaMemcpyAsync(lb, crown_lb, (size_t)B * nspec * 4, cudaMemcpyDeviceToDevice, s));
            LB_CUDA(cudaMemcpyAsync(ub, crown_ub, (size_t)B * nspec * 4, cudaMemcpyDeviceToDevice, s));
            return;
        }
    } else {
        const std::vector<int> ones(B, 1);
        LB_CUDA(cudaMemcpyAsync(bc.active, ones.data(), B * 4, cudaMemcpyHostToDevice, s));
    }
    LB_CUDA(cudaMemcpyAsync(active0, bc.active, B * 4, cudaMemcpyDeviceToDevice, s));
    alpha_ = true;
    bc.best = cache_.as<float>("ctl_best", (size_t)B * nspec);
    bc.best_loss = cache_.as<float>("ctl_bestloss", B);
    bc.patience = cache_.as<int>("ctl_pat", B);
    bc.has_best = cache_.as<int>("ctl_hasbest", B);
    bc.save = cache_.as<int>("ctl_save", B);
    bc.improved = cache_.as<uint8_t>("ctl_improved", (size_t)B * nspec);
    bc.first_save = cache_.as<int>("ctl_first", B);
    if (thr_ && opt_.stop_alpha_on_verified) {
        bc.thr = thr_;
        bc.branch = branch_;
        bc.n_branches = n_branches_;
    }
    // With thresholds, boxes stop early; the loop ends once none is left.
    int* n_active = thr_ ? cache_.as<int>("ctl_nactive", 1) : nullptr;
    bc.n_active = n_active;
    const int iters = (int)opt_.alpha_iterations;
    const int save_after = (int)((float)iters * opt_.start_save_best);
    float* cur_lb = cache_.as<float>("cur_lb", (size_t)B * nspec);
    float* cur_ub = cache_.as<float>("cur_ub", (size_t)B * nspec);
    float* neg_ub = opt_upper ? cache_.as<float>("neg_ub", (size_t)B * nspec) : nullptr;
    float* fin_lb = cache_.as<float>("fin_lb", (size_t)B * nspec);
    float* fin_ub = cache_.as<float>("fin_ub", (size_t)B * nspec);
    float* gout = cache_.as<float>(key("g", K_), std::max(2 * out.rows.R, 1));
    // TorchModel::runAlphaCROWN (:838-850): the upper side is optimised first,
    // then the lower side, in one AlphaCROWNAnalysis: the lower run starts from
    // the alphas the upper run left (its best ones), with a new Adam state,
    // learning rate and best-bound bookkeeping (computeOptimizedBounds,
    // AlphaCROWNAnalysis.cpp:306-511, each call).
    std::vector<bool> sides;
    if (opt_upper) sides.push_back(true);
    if (opt_lower) sides.push_back(false);
    int it = 0;
    for (size_t run = 0; run < sides.size(); ++run) {
        const bool up = sides[run];
        if (run > 0) LB_CUDA(cudaMemcpyAsync(bc.active, active0, B * 4, cudaMemcpyDeviceToDevice, s));
        // First pass of the run: alphas created from the CROWN slopes in the
        // first run, reused in the second; no STE reference bounds yet.
        run_pass(run == 0 ? Pass::ALPHA_FIRST : Pass::ALPHA_RESTART, B, nspec, s);
        for (int m = 1; m < K_; ++m) {
            const size_t bn = (size_t)B * width(m) * 4;
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_l", m), bn / 4), cache_.as<float>(key("cur_l", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
            LB_CUDA(cudaMemcpyAsync(cache_.as<float>(key("best_u", m), bn / 4), cache_.as<float>(key("cur_u", m), bn / 4),
                                    bn, cudaMemcpyDeviceToDevice, s));
        }
        launch_fill_f32(bc.best_loss, INFINITY, B, s);
        LB_CUDA(cudaMemsetAsync(bc.patience, 0, B * 4, s));
        LB_CUDA(cudaMemsetAsync(bc.has_best, 0, B * 4, s));
        LB_CUDA(cudaMemsetAsync(bc.save, 0, B * 4, s));
        const std::vector<int> ones(B, 1);
        LB_CUDA(cudaMemcpyAsync(bc.first_save, ones.data(), B * 4, cudaMemcpyHostToDevice, s));
        for (int st = 2; st <= K_; ++st)
            for (int m = 1; m < st; ++m) {
                const size_t cnt = (size_t)2 * starts_[st].rows.R * rowlen(st, m);
                LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("am", m, st), cnt), 0, cnt * 4, s));
                LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("av", m, st), cnt), 0, cnt * 4, s));
            }
        float lr = opt_.alpha_lr;
        int steps = 0;
        for (it = 0; it < iters; ++it) {
            const bool last = it == iters - 1;
            run_pass(Pass::ALPHA_ITER, B, nspec, s);
            val_out = cache_.as<float>(key("val", K_), (size_t)2 * out.rows.R);
            launch_scatter_output(out.rows, val_out, nspec, up, cur_lb, cur_ub, s);
            if (n_active) LB_CUDA(cudaMemsetAsync(n_active, 0, sizeof(int), s));
            if (up) {
                // Minimising ub is maximising -ub (see launch_alpha_control).
                launch_negate(cur_ub, neg_ub, (int64_t)B * nspec, s);
                launch_alpha_control(bc, neg_ub, cur_lb, B, nspec, it, save_after, (int)opt_.early_stop_patience,
                                     !last, s);
            } else {
                launch_alpha_control(bc, cur_lb, nullptr, B, nspec, it, save_after, (int)opt_.early_stop_patience,
                                     !last, s);
            }
            for (int m = 1; m < K_; ++m) {
                const size_t bn = (size_t)B * width(m);
                launch_snapshot(bc.save, cache_.as<float>(key("cur_l", m), bn), cache_.as<float>(key("cur_u", m), bn),
                                B, width(m), cache_.as<float>(key("best_l", m), bn),
                                cache_.as<float>(key("best_u", m), bn), s);
            }
            // updateBestAlphas: every active box saves at iteration 0 (nothing is
            // best yet, so every spec improves), which is each box's first save
            // and copies every row; later saves copy only rows whose index inside
            // the box is an improved spec index.
            for (int st = 2; st <= K_; ++st)
                for (int m = 1; m < st; ++m) {
                    const size_t cnt = (size_t)2 * starts_[st].rows.R * rowlen(st, m);
                    float* a = cache_.as<float>(key("alpha", m, st), cnt);
                    float* best_a = cache_.as<float>(key("abest", m, st), cnt);
                    if (it == 0)
                        LB_CUDA(cudaMemcpyAsync(best_a, a, cnt * 4, cudaMemcpyDeviceToDevice, s));
                    else
                        launch_best_alpha_rows(starts_[st].rows, B, bc.save, bc.improved, nspec, rowlen(st, m), a,
                                               best_a, s);
                }
            launch_clear_first_save(bc.save, bc.first_save, B, s);
            if (last) break;
            if (n_active) {
                // Later iterations change nothing for a box that has stopped, so
                // once every box has stopped the loop can end.
                int h_active = 0;
                LB_CUDA(cudaMemcpyAsync(&h_active, n_active, sizeof(int), cudaMemcpyDeviceToHost, s));
                LB_CUDA(cudaStreamSynchronize(s));
                if (h_active == 0) break;
            }
            // --- hand-written adjoint of the whole pass (replaces loss.backward())
            // with the torch::optim::Adam step + [0, 1] clip fused into it ---------
            for (int m = 1; m < K_; ++m) {
                const size_t bn = (size_t)B * width(m);
                LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("kbar", m), bn), 0, bn * 4, s));
                LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("bbar", m), bn), 0, bn * 4, s));
                if (act_[m] == ACT_SIGMOID) {
                    LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("sbar", m), bn), 0, bn * 4, s));
                    LB_CUDA(cudaMemsetAsync(cache_.as<float>(key("blbar", m), bn), 0, bn * 4, s));
                }
            }
            ++steps;
            adam_active_ = bc.active;
            adam_step_ = (float)((double)lr / (1.0 - std::pow(0.9, steps)));
            adam_bc2_sqrt_ = (float)std::sqrt(1.0 - std::pow(0.999, steps));
            if (up) {
                // loss = sum ub: the upper rows of the output start, seed +1.
                launch_output_seed_upper(out.rows, bc.active, gout, s);
                adjoint_start(out, B, gout, 2 * out.rows.R, s);
            } else {
                launch_output_seed(out.rows, bc.active, gout, s);
                adjoint_start(out, B, gout, out.rows.R, s);
            }
            for (int st = K_ - 1; st >= 2; --st) {
                StartPlan& sp = starts_[st];
                if (sp.rows.R == 0) continue;
                const size_t bn = (size_t)B * width(st);
                float* g = cache_.as<float>(key("g", st), (size_t)2 * sp.rows.R);
                if (act_[st] == ACT_SIGMOID)
                    launch_sigmoid_bound_grad(sp.rows, cache_.as<float>(key("cur_l", st), bn),
                                              cache_.as<float>(key("cur_u", st), bn),
                                              cache_.as<float>(key("sbar", st), bn),
                                              cache_.as<float>(key("blbar", st), bn),
                                              cache_.as<float>(key("kbar", st), bn),
                                              cache_.as<float>(key("bbar", st), bn), width(st), g, s);
                else
                    launch_bound_grad(sp.rows, cache_.as<float>(key("cur_l", st), bn),
                                      cache_.as<float>(key("cur_u", st), bn), cache_.as<uint8_t>(key("rp_f", st), bn),
                                      cache_.as<float>(key("kbar", st), bn), cache_.as<float>(key("bbar", st), bn),
                                      width(st), g, s);
                adjoint_start(sp, B, g, 2 * sp.rows.R, s);
            }
            lr = lr * opt_.alpha_lr_decay;
        }
        // --- restoreBestAlphas, restoreBestIntermediateBounds, final run(false) ---
        for (int st = 2; st <= K_; ++st)
            for (int m = 1; m < st; ++m) {
                const size_t cnt = (size_t)2 * starts_[st].rows.R * rowlen(st, m);
                // A seeded box's best alphas are its alphas themselves
                // (seedAlphas: _bestAlphaByNodeStart = _alphaByNodeStart), so
                // restoring leaves them as they are.
                launch_restore_alpha(starts_[st].rows, bc.first_save, rowlen(st, m),
                                     cache_.as<float>(key("abest", m, st), cnt),
                                     cache_.as<float>(key("alpha", m, st), cnt), s,
                                     warm_on_ ? cache_.as<int>(key("wseed", st), B) : nullptr);
            }
        run_pass(Pass::ALPHA_FINAL, B, nspec, s);
        val_out = cache_.as<float>(key("val", K_), (size_t)2 * out.rows.R);
        if (up) {
            // Upper: min(final, best).  A lower side that is not optimised is
            // the runCROWN that follows (:858-862), over the same nodes: the
            // lower side of this pass.
            launch_scatter_output(out.rows, val_out, nspec, true, fin_lb, fin_ub, s);
            launch_negate(fin_ub, neg_ub, (int64_t)B * nspec, s);
            launch_max_best(bc.best, bc.has_best, B * nspec, nspec, neg_ub, s);
            launch_negate(neg_ub, ub, (int64_t)B * nspec, s);
            if (!opt_lower) LB_CUDA(cudaMemcpyAsync(lb, fin_lb, (size_t)B * nspec * 4, cudaMemcpyDeviceToDevice, s));
        } else {
            // Lower: max(final, best).  An upper side that is not optimised
            // comes from the runCROWN that follows, over the same nodes (same
            // best intermediate bounds and alphas): the upper side of this pass.
            launch_scatter_output(out.rows, val_out, nspec, upper && !opt_upper, lb, ub, s);
            launch_max_best(bc.best, bc.has_best, B * nspec, nspec, lb, s);
        }
        iters_run_ = std::max(iters_run_, std::min(it + 1, iters));
    }
    if (done) launch_take_verified(done, crown_lb, crown_ub, B, nspec, lb, ub, s);
    if (warm_keep_) {
        if (!opt_upper && !has_sigmoid_ && !thr_)
            warm_retain(B, s);
        else
            warm_valid_ = false;
    }
    (void)nout;
}

// The tensor-core schedule needs every contraction shape on the tensor-core
// path: all widths that appear as N or K of a contraction (n_0 .. n_{K-1})
// multiples of 16.
bool Model::tc_eligible() const {
    if (force_simt_ || has_conv_ || has_sigmoid_) return false;
    for (int m = 0; m < K_; ++m)
        if (!tc_supported(1, width(m), width(m)) || width(m) % 16 != 0) return false;
    return true;
}

// ------------------------------------------------------------ profiling
void Model::prof_begin(cudaStream_t s) {
    if (!profile_) return;
    while (ev_pool_.size() < ev_used_ + 2) {
        cudaEvent_t e;
        LB_CUDA(cudaEventCreate(&e));
        ev_pool_.push_back(e);
    }
    LB_CUDA(cudaEventRecord(ev_pool_[ev_used_], s));
}

void Model::prof_end(cudaStream_t s, double flops) {
    if (!profile_) return;
    LB_CUDA(cudaEventRecord(ev_pool_[ev_used_ + 1], s));
    ev_used_ += 2;
    contraction_flops_ += flops;
    ++contraction_launches_;
}

// Sum of the recorded contraction intervals (the stream has been synchronised).
double Model::prof_collect() {
    double ms = 0.0;
    for (size_t i = 0; i + 1 < ev_used_; i += 2) {
        float t = 0.f;
        LB_CUDA(cudaEventElapsedTime(&t, ev_pool_[i], ev_pool_[i + 1]));
        ms += t;
    }
    ev_used_ = 0;
    return ms;
}

// ------------------------------------------------------------ entry
void Model::compute(int method, const float* d_xl, const float* d_xu, int64_t n_boxes, const float* d_C,
                    int64_t c_boxes, int64_t nspec, const float* d_thr, bool lower, bool upper,
                    float* d_lb, float* d_ub, cudaStream_t stream, lb200_stats* stats, const int32_t* d_branch,
                    int n_branches) {
    (void)lower;
    if (method < LB200_METHOD_IBP || method > LB200_METHOD_ALPHA_CROWN) throw std::invalid_argument("unknown method");
    if (n_boxes < 0 || nspec <= 0) throw std::invalid_argument("bad sizes");
    if (c_boxes != 1 && c_boxes != n_boxes) throw std::invalid_argument("c_boxes must be 1 or n_boxes");
    if (n_branches < 0 || (n_branches > 0 && (!d_branch || !d_thr)))
        throw std::invalid_argument("OR branches need thresholds and a branch index per row");
    // Warm start: parents set by set_warm_parents apply to this call only.
    const bool warm = warm_pending_;
    warm_pending_ = false;
    if (warm) {
        if (method != LB200_METHOD_ALPHA_CROWN) throw std::invalid_argument("warm start: alpha-CROWN calls only");
        if ((int64_t)warm_parent_.size() != n_boxes)
            throw std::invalid_argument("warm start: one parent index per box is needed");
        if (has_sigmoid_) throw std::invalid_argument("warm start: networks with Sigmoid are not supported");
        if (d_thr) throw std::invalid_argument("warm start: specification thresholds are not supported");
        if (upper && opt_.optimize_upper) throw std::invalid_argument("warm start: OPTIMIZE_UPPER is not supported");
    }
    // A call that fails after this point leaves no retained state behind.
    struct WarmReset {
        Model* m;
        bool ok = false;
        ~WarmReset() {
            m->warm_on_ = false;
            if (!ok && m->warm_keep_) m->warm_valid_ = false;
        }
    } warm_reset{this};
    // What warm start does not cover leaves no retained state.
    if (warm_keep_ && method == LB200_METHOD_ALPHA_CROWN &&
        (d_thr || has_sigmoid_ || (upper && opt_.optimize_upper)))
        warm_valid_ = false;
    thr_ = d_thr;
    branch_ = d_branch;
    n_branches_ = n_branches;
    iters_run_ = 0;
    LB_CUDA(cudaSetDevice(device_));
    const auto t0 = std::chrono::steady_clock::now();
    launch_counter() = 0;
    ev_used_ = 0;
    contraction_flops_ = 0.0;
    contraction_launches_ = 0;
    flops_ = 0.0;
    rows_ = 0;
    cudaEvent_t e0, e1;
    LB_CUDA(cudaEventCreate(&e0));
    LB_CUDA(cudaEventCreate(&e1));
    LB_CUDA(cudaEventRecord(e0, stream));
    const bool alpha = method == LB200_METHOD_ALPHA_CROWN;
    size_t free_b = 0, total_b = 0;
    LB_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const size_t budget = (size_t)((double)(free_b + cache_.total_bytes()) * 0.7);
    const int64_t per_box = std::max<int64_t>(1, (int64_t)bytes_per_box(alpha, (int)nspec));
    int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(n_boxes, (int64_t)(budget / per_box)));
    chunk = std::min<int64_t>(chunk, 65536);
    if (warm) {
        if (chunk < n_boxes)
            throw std::invalid_argument("warm start: the boxes do not fit one chunk on this device");
        LB_CUDA(cudaMemcpyAsync(cache_.as<int>("wparent", std::max<int64_t>(n_boxes, 1)), warm_parent_.data(),
                                (size_t)n_boxes * sizeof(int), cudaMemcpyHostToDevice, stream));
        warm_on_ = n_boxes > 0;
    }
    const int n0 = n_in(), nout = n_out();
    for (int64_t b0 = 0; b0 < n_boxes; b0 += chunk) {
        const int B = (int)std::min<int64_t>(chunk, n_boxes - b0);
        const float* C = d_C + (c_boxes == 1 ? 0 : b0 * nspec * nout);
        run_chunk(method, d_xl + b0 * n0, d_xu + b0 * n0, B, C, c_boxes == 1 ? 0 : 1, (int)nspec, upper,
                  d_lb + b0 * nspec, d_ub + b0 * nspec, stream);
        last_B_ = B;
    }
    last_alpha_ = alpha;
    // Retained state covers one chunk: a call split into several keeps none.
    if (warm_keep_ && n_boxes > chunk) warm_valid_ = false;
    LB_CUDA(cudaEventRecord(e1, stream));
    LB_CUDA(cudaEventSynchronize(e1));
    int tc_err = 0;
    LB_CUDA(cudaMemcpy(&tc_err, tc_error_flag(), sizeof(int), cudaMemcpyDeviceToHost));
    if (tc_err) {
        LB_CUDA(cudaMemset(tc_error_flag(), 0, sizeof(int)));
        throw std::runtime_error("tensor-core contraction: a bounded wait expired; results are invalid");
    }
    warm_reset.ok = true;
    float ms = 0.f;
    LB_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (stats) {
        stats->ms_device = ms;
        stats->ms_total = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        stats->kernel_launches = launch_counter();
        stats->backward_rows = rows_;
        stats->algorithmic_flops = flops_;
        stats->alpha_iterations_run = alpha ? iters_run_ : 0;
        stats->ms_contractions = prof_collect();
        stats->contraction_launches = contraction_launches_;
        stats->contraction_flops = contraction_flops_;
    }
}

int64_t Model::intermediate_count() const {
    int64_t t = 0;
    for (int m = 1; m < K_; ++m) t += width(m);
    return t * last_B_;
}

void Model::copy_intermediate(float* lower, float* upper) const {
    // Per box, pre-activations in the node-id order of the nodes that hold them.
    const int B = last_B_;
    int64_t per = 0;
    for (int m = 1; m < K_; ++m) per += width(m);
    std::vector<int> lv;
    for (int m = 1; m < K_; ++m) lv.push_back(m);
    std::sort(lv.begin(), lv.end(),
              [&](int a, int b) { return preact_node_ids_[a - 1] < preact_node_ids_[b - 1]; });
    std::vector<float> tmp;
    int64_t off = 0;
    for (int m : lv) {
        const int n = width(m);
        tmp.resize((size_t)B * n);
        for (int side = 0; side < 2; ++side) {
            const char* nm = last_alpha_ ? (side ? "best_u" : "best_l") : (side ? "cur_u" : "cur_l");
            const void* src = const_cast<DevCache&>(cache_).get(key(nm, m), (size_t)B * n * 4);
            LB_CUDA(cudaMemcpy(tmp.data(), src, (size_t)B * n * 4, cudaMemcpyDeviceToHost));
            float* dst = side ? upper : lower;
            const MapShape& ms = map(m);
            if (ms.spatial) {
                // HWC -> Luna's CHW order.
                const int HW = ms.H * ms.W;
                for (int b = 0; b < B; ++b)
                    for (int i = 0; i < n; ++i)
                        dst[b * per + off + (i % ms.C) * HW + i / ms.C] = tmp[(size_t)b * n + i];
            } else {
                for (int b = 0; b < B; ++b) std::memcpy(dst + b * per + off, tmp.data() + (size_t)b * n, n * 4);
            }
        }
        off += n;
    }
}

}  // namespace lb200
