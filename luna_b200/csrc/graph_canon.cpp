// graph_canon.cpp -- see graph_canon.h.
#include "graph_canon.h"

#include <algorithm>
#include <cstdint>
#include <stdexcept>

namespace lb200 {

namespace {

int64_t numel(const lb200_node_desc& d) { return (int64_t)d.out_shape[0] * d.out_shape[1] * d.out_shape[2]; }

bool flat(const lb200_node_desc& d) { return d.out_shape[1] == 1 && d.out_shape[2] == 1; }

// ONNX's "negative infinity" end of a reversed slice.
constexpr int64_t kNegInf = -9223372036854775807LL;

}  // namespace

CanonGraph canonicalize(const lb200_graph_desc* g) {
    if (!g || g->num_nodes <= 0 || !g->nodes) throw std::invalid_argument("empty graph");
    CanonGraph cg;
    const int n = g->num_nodes;
    cg.nodes.assign(g->nodes, g->nodes + n);
    cg.dead.assign(n, 0);
    auto& N = cg.nodes;
    auto bad = [&](int i, const std::string& why) {
        throw std::invalid_argument("node " + std::to_string(i) + " (type " + std::to_string(N[i].type) + "): " + why);
    };
    auto keep = [&](std::vector<float> v) -> const float* {
        cg.store.push_back(std::make_unique<std::vector<float>>(std::move(v)));
        return cg.store.back()->data();
    };
    // Consumers of every node (ids in ascending order).
    auto consumers = [&](int p) {
        std::vector<int> c;
        for (int i = 0; i < n; ++i) {
            if (cg.dead[i]) continue;
            for (int k = 0; k < N[i].num_inputs; ++k)
                if (N[i].inputs[k] == p) {
                    c.push_back(i);
                    break;
                }
        }
        return c;
    };
    auto check_inputs = [&](int i) {
        const auto& d = N[i];
        if (d.num_inputs < 0 || d.num_inputs > 4) bad(i, "bad num_inputs");
        for (int k = 0; k < d.num_inputs; ++k)
            if (d.inputs[k] < 0 || d.inputs[k] >= n) bad(i, "bad input index");
    };
    auto sole_consumer = [&](int p, int i) {
        const auto c = consumers(p);
        return c.size() == 1 && c[0] == i && p != g->output_index;
    };
    for (int i = 0; i < n; ++i) check_inputs(i);

    bool any = false;
    for (int i = 0; i < n; ++i) {
        const int t = N[i].type;
        if (t == LB200_NODE_RESHAPE || t == LB200_NODE_SUB || t == LB200_NODE_SLICE || t == LB200_NODE_CONCAT) {
            any = true;
            break;
        }
    }
    // Nodes are visited in id order; a rewrite only looks at producers, which
    // (in a graph a front end builds) have smaller ids.  Producers with a
    // larger id are rejected below.
    for (int i = 0; any && i < n; ++i) {
        lb200_node_desc& d = N[i];
        for (int k = 0; k < d.num_inputs; ++k)
            if (d.inputs[k] >= i &&
                (d.type == LB200_NODE_RESHAPE || d.type == LB200_NODE_SUB || d.type == LB200_NODE_SLICE ||
                 d.type == LB200_NODE_CONCAT))
                bad(i, "producers must precede the node");
        switch (d.type) {
        case LB200_NODE_RESHAPE: {
            // Luna's Reshape flattens (ReshapeWrapper with shape -1, batch kept).
            if (d.num_inputs != 1) bad(i, "Reshape expects one input");
            const auto& p = N[d.inputs[0]];
            if (numel(d) != numel(p)) bad(i, "Reshape changes the number of features");
            if (!flat(d)) bad(i, "Reshape to a map is not supported (Luna's Reshape flattens)");
            d.type = LB200_NODE_FLATTEN;
            break;
        }
        case LB200_NODE_SUB: {
            if (d.num_inputs != 1) bad(i, "Sub of two tensors is not supported");
            if (!d.constant) bad(i, "Sub without a constant");
            const int pi = d.inputs[0];
            lb200_node_desc& p = N[pi];
            if (numel(d) != numel(p)) bad(i, "Sub output size differs from its input");
            const int64_t m = numel(p);
            const bool neg = d.constant_second == 0;
            if (p.type == LB200_NODE_INPUT) {
                if (!sole_consumer(pi, i)) bad(i, "a Sub on the input must be the input's only consumer");
                if (cg.in_tf) bad(i, "a second Sub on the input");
                cg.in_tf = true;
                cg.in_neg = neg;
                cg.in_const.assign(d.constant, d.constant + m);
                d.type = LB200_NODE_IDENTITY;
                break;
            }
            if ((p.type != LB200_NODE_LINEAR && p.type != LB200_NODE_CONV) || !sole_consumer(pi, i))
                bad(i, "Sub must follow the input, or a Linear / Conv node it alone consumes");
            if (!p.weight) bad(pi, "affine node without weight");
            const int nch = p.out_shape[0];
            const int64_t hw = (int64_t)p.out_shape[1] * p.out_shape[2];
            std::vector<float> cch(nch);
            for (int c = 0; c < nch; ++c) {
                cch[c] = d.constant[(int64_t)c * hw];
                for (int64_t q = 1; q < hw; ++q)
                    if (d.constant[(int64_t)c * hw + q] != cch[c])
                        bad(i, "a Sub after a Conv needs a constant uniform over each channel");
            }
            std::vector<float> b(nch, 0.f);
            if (p.bias)
                for (int c = 0; c < nch; ++c) b[c] = p.bias[c];
            const int64_t wn = p.type == LB200_NODE_LINEAR ? (int64_t)p.out_features * p.in_features
                                                            : (int64_t)nch * N[p.inputs[0]].out_shape[0] *
                                                                  p.kernel[0] * p.kernel[1];
            lb200_node_desc r = p;
            if (neg) {
                // c - (W x + b) = (-W) x + (c - b)
                std::vector<float> w(p.weight, p.weight + wn);
                for (auto& v : w) v = -v;
                for (int c = 0; c < nch; ++c) b[c] = cch[c] - b[c];
                r.weight = keep(std::move(w));
            } else {
                for (int c = 0; c < nch; ++c) b[c] = b[c] - cch[c];
            }
            r.bias = keep(std::move(b));
            d = r;  // node i becomes the folded affine node, reading p's producer
            cg.dead[pi] = 1;
            break;
        }
        case LB200_NODE_SLICE: {
            if (d.num_inputs != 1) bad(i, "Slice expects one input");
            const int pi = d.inputs[0];
            lb200_node_desc& p = N[pi];
            if (!flat(p) || d.axis != 1) bad(i, "only slices along the features of a flat vector are supported");
            const int64_t len_in = numel(p);
            if (d.step != 1 && d.step != -1) bad(i, "Slice steps other than 1 and -1 are not supported");
            // BoundedSliceNode::_fixup_params (BoundedSliceNode.cpp:28-52).
            int64_t a = d.start, e = d.end;
            if (a < 0) a += len_in;
            if (e < 0) e = e == kNegInf ? 0 : e + len_in;
            if (d.step == -1) {
                std::swap(a, e);
                e = e + 1;
            }
            e = std::min(e, len_in);
            a = std::max<int64_t>(a, 0);
            const int64_t len = e - a;
            if (len <= 0) bad(i, "empty slice");
            if (numel(d) != len) bad(i, "Slice out_shape does not match its range");
            // Output feature j is input feature idx(j).
            auto idx = [&](int64_t j) { return d.step == 1 ? a + j : e - 1 - j; };
            if (p.type == LB200_NODE_LINEAR && sole_consumer(pi, i)) {
                if (!p.weight) bad(pi, "Linear without weight");
                std::vector<float> w((size_t)len * p.in_features), b((size_t)len, 0.f);
                for (int64_t j = 0; j < len; ++j) {
                    std::copy(p.weight + idx(j) * p.in_features, p.weight + (idx(j) + 1) * p.in_features,
                              w.begin() + j * p.in_features);
                    if (p.bias) b[j] = p.bias[idx(j)];
                }
                lb200_node_desc r = p;
                r.out_features = len;
                r.out_shape[0] = (int32_t)len;
                r.out_shape[1] = r.out_shape[2] = 1;
                r.weight = keep(std::move(w));
                r.bias = keep(std::move(b));
                d = r;
                cg.dead[pi] = 1;
                break;
            }
            // Every consumer a Linear: widen it with zero columns and read p.
            const auto cons = consumers(i);
            if (cons.empty() || i == g->output_index) bad(i, "a Slice must feed Linear nodes or follow a Linear");
            for (int c : cons) {
                lb200_node_desc& q = N[c];
                if (q.type != LB200_NODE_LINEAR || q.num_inputs != 1 || !q.weight || q.in_features != len)
                    bad(i, "a Slice must feed Linear nodes or follow a Linear");
                std::vector<float> w((size_t)q.out_features * len_in, 0.f);
                for (int64_t o = 0; o < q.out_features; ++o)
                    for (int64_t j = 0; j < len; ++j) w[o * len_in + idx(j)] = q.weight[o * len + j];
                q.weight = keep(std::move(w));
                q.in_features = len_in;
                q.inputs[0] = pi;
            }
            cg.dead[i] = 1;
            break;
        }
        case LB200_NODE_CONCAT: {
            if (d.num_inputs < 2) bad(i, "Concat expects at least two inputs");
            if (d.axis != 1) bad(i, "only Concat along axis 1 (features / channels) is supported");
            const int t0 = N[d.inputs[0]].type;
            const int src = N[d.inputs[0]].num_inputs == 1 ? N[d.inputs[0]].inputs[0] : -1;
            for (int k = 0; k < d.num_inputs; ++k) {
                const int pi = d.inputs[k];
                const auto& p = N[pi];
                if ((p.type != LB200_NODE_LINEAR && p.type != LB200_NODE_CONV) || p.type != t0 ||
                    p.num_inputs != 1 || p.inputs[0] != src || !p.weight || !sole_consumer(pi, i))
                    bad(i, "Concat operands must be Linear (or Conv) nodes of one producer, consumed only here");
                for (int k2 = 0; k2 < k; ++k2)
                    if (d.inputs[k2] == pi) bad(i, "a Concat operand repeated");
            }
            lb200_node_desc r = N[d.inputs[0]];
            std::vector<float> w, b;
            int64_t rows = 0;
            if (t0 == LB200_NODE_LINEAR) {
                for (int k = 0; k < d.num_inputs; ++k) {
                    const auto& p = N[d.inputs[k]];
                    if (p.in_features != r.in_features) bad(i, "Concat of Linear nodes with different inputs");
                    // The Gemm scale of each operand is applied to its rows
                    // here, exactly as the engine applies it at build time.
                    for (int64_t q = 0; q < p.out_features * p.in_features; ++q) w.push_back(p.scale * p.weight[q]);
                    for (int64_t o = 0; o < p.out_features; ++o) b.push_back(p.bias ? p.bias[o] : 0.f);
                    rows += p.out_features;
                }
                r.scale = 1.0f;
                r.out_features = rows;
                r.out_shape[0] = (int32_t)rows;
                r.out_shape[1] = r.out_shape[2] = 1;
            } else {
                for (int k = 0; k < d.num_inputs; ++k) {
                    const auto& p = N[d.inputs[k]];
                    for (int a = 0; a < 2; ++a)
                        if (p.kernel[a] != r.kernel[a] || p.stride[a] != r.stride[a] || p.padding[a] != r.padding[a])
                            bad(i, "Concat of Conv nodes with different geometry");
                    if (p.out_shape[1] != r.out_shape[1] || p.out_shape[2] != r.out_shape[2])
                        bad(i, "Concat of Conv maps of different sizes");
                    const int64_t per = (int64_t)N[src].out_shape[0] * p.kernel[0] * p.kernel[1];
                    w.insert(w.end(), p.weight, p.weight + (int64_t)p.out_shape[0] * per);
                    for (int c = 0; c < p.out_shape[0]; ++c) b.push_back(p.bias ? p.bias[c] : 0.f);
                    rows += p.out_shape[0];
                }
                r.out_shape[0] = (int32_t)rows;
            }
            if (numel(d) != numel(r)) bad(i, "Concat out_shape does not match its operands");
            r.weight = keep(std::move(w));
            r.bias = keep(std::move(b));
            for (int k = 0; k < d.num_inputs; ++k) cg.dead[d.inputs[k]] = 1;
            d = r;
            break;
        }
        default:
            break;
        }
    }
    // Nodes without a path to the output are dead.
    if (g->output_index < 0 || g->output_index >= n) throw std::invalid_argument("bad output_index");
    std::vector<char> live(n, 0);
    std::vector<int> work{g->output_index};
    live[g->output_index] = 1;
    while (!work.empty()) {
        const int c = work.back();
        work.pop_back();
        for (int k = 0; k < N[c].num_inputs; ++k) {
            const int p = N[c].inputs[k];
            if (!live[p]) {
                live[p] = 1;
                work.push_back(p);
            }
        }
    }
    for (int i = 0; i < n; ++i) cg.dead[i] = !live[i];
    if (!live[g->input_index]) throw std::invalid_argument("the output does not depend on the input");
    cg.desc.num_nodes = n;
    cg.desc.nodes = cg.nodes.data();
    cg.desc.input_index = g->input_index;
    cg.desc.output_index = g->output_index;
    return cg;
}

}  // namespace lb200
