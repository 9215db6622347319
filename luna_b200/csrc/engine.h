// engine.h -- host side of the luna_b200 engine.
//
// A Model holds one network on one GPU and bounds batches of input boxes
// with IBP, CROWN or alpha-CROWN, each box exactly as Luna bounds it on a
// fresh TorchModel (src/engine/TorchModel.cpp:653-698).
#pragma once

#include "../../include/luna_b200.h"
#include "conv_kernels.cuh"
#include "kernels.cuh"
#include "tc_conv.cuh"

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace lb200 {

// Grow-only cache of named device buffers owned by a model.
class DevCache {
public:
    ~DevCache();
    void* get(const std::string& name, size_t bytes);
    template <class T>
    T* as(const std::string& name, size_t count) {
        return static_cast<T*>(get(name, count * sizeof(T)));
    }
    size_t total_bytes() const;
    size_t capacity(const std::string& name) const;
    void release();

private:
    struct Buf {
        void* p = nullptr;
        size_t bytes = 0;
    };
    std::map<std::string, Buf> bufs_;
};

// Shape of the feature map at one level (the output of layer m, or the
// input for m = 0).  Maps next to a conv layer are "spatial" and stored HWC;
// the others are flat vectors (C = n, H = W = 1).
struct MapShape {
    int C = 1, H = 1, W = 1;
    bool spatial = false;
    int n() const { return C * H * W; }
};

// One affine layer: Linear (BoundedLinearNode) or Conv2d (BoundedConvNode).
struct Layer {
    bool conv = false;
    bool convt = false;  // ConvTranspose2d (BoundedConvTransposeNode): W = Wg [Ci][kh][kw][Co], Wt = Wa [kh][kw][Co][Ci]
    int n_in = 0, n_out = 0;
    MapShape in, out;
    int kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0;  // conv geometry
    // Linear: W [n_out, n_in] and Wt [n_in, n_out], input columns in the
    // engine's feature order (HWC after a Flatten of a conv map).
    // Conv: W = Wc [Co][kh][kw][Ci], Wt = Wk [kh][kw][Co][Ci].
    float* W = nullptr;
    float* Wt = nullptr;
    float* b = nullptr;        // [n_out] (Linear) or [Co] (conv)
    std::vector<float> b_host; // the same bias on the host
    float* b_neuron = nullptr; // [n_out]: bias of every output neuron
    // tf32 (hi, lo) splits for the tensor-core path (Linear): W is the K-major
    // B operand of the adjoint contraction, Wt of the forward one.
    float *W_hi = nullptr, *W_lo = nullptr, *Wt_hi = nullptr, *Wt_lo = nullptr;
    // Tensor-core conv weights (weights-stationary implicit GEMM, tf32 hi/lo):
    // forward (transposed conv) Wf [s*s*Ci, Uy*Ux*Co], rows (phase, ci), K
    // blocks (u_y, u_x, co block); adjoint (correlation) Wa [Co, |adj_kb|*32],
    // K blocks (phase, u_y, u_x, ci block) for the taps that exist.
    bool tcf = false, tca = false;
    int Uy = 0, Ux = 0;
    float *Wf_hi = nullptr, *Wf_lo = nullptr, *Wa_hi = nullptr, *Wa_lo = nullptr;
    std::vector<TcConvTap> adj_kb;  // plane, u_y (dy), u_x (dx), c0
    // Tensor-core steps of a ConvTranspose2d layer (same kernel kinds with
    // the roles of the two sides swapped): back-substitution as a strided
    // correlation, Wtb [Ci, |tcb_kb| * 32], K blocks (tap, co block) reading
    // A at (q s - p + k); adjoint as a transposed conv with the s*s phases
    // stacked in M, Wtj [s*s*Co, Uy*Ux*Ci], K blocks (u_y, u_x, ci block).
    bool tct_b = false, tct_a = false;
    float *Wtb_hi = nullptr, *Wtb_lo = nullptr, *Wtj_hi = nullptr, *Wtj_lo = nullptr;
    std::vector<TcConvTap> tcb_kb;
};

// A skip edge into the Add at a level: from the ReLU output of level `src`,
// directly (identity) or through a conv (L, BatchNorm folded).
struct SkipEdge {
    int src = 0;
    int node = -1, bn = -1;  // graph node ids (-1: identity / no BatchNorm)
    std::shared_ptr<Layer> L;
};

struct StartPlan {
    int s = 0;          // pre-activation index (1..K-1), or K for the output start
    RowMap rows;        // device row map (R rows per side)
    int* row_box = nullptr;
    int* row_id = nullptr;
    int* box_off = nullptr;
    // Row geometry at every level up to the start (index m = 0 .. s):
    // windows for a conv start, whole maps otherwise.
    std::vector<WinGeo> geo;
    int form = CONC_DENSE;  // concretisation form Luna uses for this start
};

class Model {
public:
    // on_device = false builds only the host-side plan (levels, row
    // geometry, concretisation forms) for describe(); no GPU is touched.
    Model(const lb200_graph_desc* g, int device, bool on_device = true);
    ~Model();

    void set_options(const lb200_options& o) { opt_ = o; }
    void set_profiling(bool on) { profile_ = on; }
    // Contraction path: tensor cores (3xTF32) where the shape allows, else
    // the SIMT fp32 kernel.  Forcing SIMT is for cross-checking only.
    void set_force_simt(bool on) {
        force_simt_ = on;
        tcconv_ = !on;
    }
    // Tensor-core contractions on CTA pairs (default) or on single CTAs
    // (for cross-checking).
    void set_pairs(bool on) { pairs_ = on; }
    // Adjoint contractions on the SIMT fp32 kernel while the forward ones use
    // the tensor cores (for cross-checking where precision matters).
    void set_simt_adjoint(bool on) { simt_adjoint_ = on; }
    // Tensor-core contractions with the 3xTF32 cross terms in their own TMEM
    // accumulator: the adjoint ones (default) and the forward ones.
    void set_split_acc(bool adjoint, bool forward) {
        split_adj_ = adjoint;
        split_fwd_ = forward;
    }
    // Warm start (TorchModel::getState / loadState, as branch-and-bound
    // hands a sub-domain its parent's state): with keep on, every
    // alpha-CROWN call retains its boxes' final alphas and creation sets;
    // set_warm_parents then makes the next call seed its box b from
    // retained box parent[b] (-1: bounded afresh).  Turning keep off drops
    // the retained state.
    void set_warm_keep(bool on) {
        warm_keep_ = on;
        if (!on) warm_valid_ = false;
    }
    void set_warm_parents(const int64_t* parent, int64_t n);
    // The retained alphas of one box for (activation level m, start st), both
    // sides [2, rows, cols] into out (when cap allows), and the creation set
    // [cols] into aset (when non-null); rows / cols are always set.
    void warm_alpha(int m, int st, int64_t box, float* out, int64_t cap, int64_t* rows, int64_t* cols,
                    uint8_t* aset);
    const lb200_options& options() const { return opt_; }
    // The plan as JSON: every level (node, map, activation, main edge, skip
    // edges) and every backward start (concretisation form and the row
    // window at each level below it).
    std::string describe() const;

    void compute(int method, const float* d_xl, const float* d_xu, int64_t n_boxes,
                 const float* d_C, int64_t c_boxes, int64_t nspec, const float* d_thr,
                 bool lower, bool upper, float* d_lb, float* d_ub, cudaStream_t stream,
                 lb200_stats* stats, const int32_t* d_branch = nullptr, int n_branches = 0);

    // Host-side upload helpers for the host-buffer entry point.
    float* staging(const std::string& name, size_t count) { return cache_.as<float>(name, count); }
    int device() const { return device_; }
    int n_in() const { return layers_.front().n_in; }
    int n_out() const { return layers_.back().n_out; }
    const std::vector<Layer>& layers() const { return layers_; }
    // Linear layers with ReLU between them and no joins (the networks the
    // allocation-free IBP entry point takes).
    bool is_relu_mlp() const {
        if (has_conv_ || has_sigmoid_ || in_tf_) return false;
        for (const auto& sk : skips_)
            if (!sk.empty()) return false;
        return true;
    }
    int64_t intermediate_count() const;
    void copy_intermediate(float* lower, float* upper) const;

private:
    // One bounded chunk of boxes.
    void run_chunk(int method, const float* xl, const float* xu, int B, const float* C, int c_per_box,
                   int nspec, bool upper, float* lb, float* ub, cudaStream_t s);

    // ALPHA_RESTART: the first pass of a second optimisation run (the lower
    // side after the upper one): alphas kept, no STE reference bounds.
    enum class Pass { CROWN, ALPHA_FIRST, ALPHA_ITER, ALPHA_FINAL, ALPHA_RESTART };
    void run_pass(Pass pass, int B, int nspec, cudaStream_t s);
    void forward_start(StartPlan& sp, int B, int nspec, bool save, bool alpha, cudaStream_t s);
    void adjoint_start(StartPlan& sp, int B, const float* g, int M, cudaStream_t s);
    void relu_params(int m, int B, bool alpha_mode, bool create, cudaStream_t s);
    // Relaxation parameters of level m's activation for B boxes of n neurons,
    // as the rows of start st read them (the start's own copy in a warm-started
    // call, where seeded boxes keep their parent's creation sets).
    ReluParams rview(int m, int B, int n, int st = 0);
    // Warm start: level m's relaxation per start above it, with each box's
    // creation set (its parent's where seeded) formed when `create`.
    void warm_relu_params(int m, int B, bool create, cudaStream_t s);
    // Retain this call's final alphas, creation sets and row offsets.
    void warm_retain(int B, cudaStream_t s);
    void init_alpha(StartPlan& sp, int m, int B, cudaStream_t s);
    void build_tc_conv(Layer& L, const float* w, int k);
    void build_tc_convt(Layer& L, const float* w, int k);
    // Tensor-core plans of transposed-conv layer m (whole-map rows).
    TcConvPlan tct_back_plan(int m, int rows, const float* data) const;
    TcConvPlan tct_adj_plan(int m, int rows, const float* pbar) const;
    void build_layer(Layer& L, const lb200_graph_desc* g, int node, int bn_node, const MapShape& prev, int k,
                     bool first);
    void build_geometry();
    // Skip-edge steps of level m's edge e for the rows of start st.
    SkipStep skip_step(int st, int m, int e) const;
    // Level j is the source of a skip edge into a level in (j, st] (or
    // (j, st) without the start itself).
    bool skip_source(int st, int j, bool with_start) const;
    void build_rows(int B, int nspec, cudaStream_t s);
    void alloc_alpha(int B, cudaStream_t s);
    size_t bytes_per_box(bool alpha, int nspec) const;

    int width(int m) const { return m == 0 ? layers_[0].n_in : layers_[m - 1].n_out; }
    const MapShape& map(int m) const { return m == 0 ? layers_[0].in : layers_[m - 1].out; }
    // Length of a row of start st at level m (its window, or the whole map).
    int rowlen(int st, int m) const { return geo_[st][m].size(); }
    ConvStep conv_step(int st, int m) const;
    ConvTStep convt_step(int m) const;
    // Bias that back-substitution adds for level m, per channel or per
    // neuron: the main edge's (none for a ConvTranspose: Luna's A is flat
    // there) plus every skip conv's.
    const float* level_bias(int m) const { return lvl_b_[m]; }
    const float* level_bias_n(int m) const { return lvl_bn_[m]; }
    // Tensor-core plans of conv layer m for the rows of start st.
    void conv_phase(int st, int m, int& cy, int& cx, int& tlo_y, int& tlo_x, int& nty, int& ntx) const;
    TcConvPlan tc_fwd_plan(int st, int m, int rows, const float* data) const;
    TcConvPlan tc_adj_plan(int st, int m, int rows, const float* pbar) const;
    PhaseSplit phase_split(int st, int m) const;
    bool tcconv_ = true;
    bool pairs_ = true;
    bool simt_adjoint_ = false;
    bool split_adj_ = true;
    bool split_fwd_ = false;
    int start_form(int st) const;
    bool has_conv_ = false;
    std::string key(const char* what, int a, int b = -1) const;

    int device_ = 0;
    bool on_device_ = true;
    lb200_options opt_{};
    std::vector<Layer> layers_;        // main edge into level m = layers_[m - 1], m = 1..K
    std::vector<std::vector<SkipEdge>> skips_;  // [level] skip edges into its Add
    std::vector<float*> lvl_b_, lvl_bn_;        // [level] bias of level m (level_bias)
    enum { ACT_RELU = 1, ACT_SIGMOID = 2 };
    std::vector<int> act_;                       // [level] activation (0 for the input and the output)
    bool has_sigmoid_ = false;
    std::vector<std::vector<WinGeo>> geo_;  // [start][level]
    std::vector<int> preact_node_ids_; // [m - 1] node whose output is pre-activation m (1..K-1)
    DevCache weights_;
    DevCache cache_;

    // Per-chunk state.
    int K_ = 0;
    std::vector<StartPlan> starts_;    // index s in 2..K-1 and K (output)
    const float* xl_ = nullptr;
    const float* xu_ = nullptr;
    const float* C_ = nullptr;
    int c_per_box_ = 0;
    bool alpha_ = false;
    double flops_ = 0.0;
    int64_t rows_ = 0;
    int last_B_ = 0;
    bool last_alpha_ = false;
    // Specification thresholds of the current call (device, or null) and the
    // OR branch of each row (n_branches_ == 0: a conjunction).
    const float* thr_ = nullptr;
    const int32_t* branch_ = nullptr;
    int n_branches_ = 0;
    int iters_run_ = 0;  // alpha iterations run, max over the chunks of a call

    // Sub on the input node (graph_canon.h): boxes become x - c (or c - x).
    bool in_tf_ = false;
    bool in_neg_ = false;
    float* in_const_ = nullptr;

    // Warm start: keep requested, retained state present, the current call
    // seeds from it, parents set for the next call; the retained boxes' count
    // and row totals per start; the parents of the next call's boxes.
    bool warm_keep_ = false;
    bool warm_valid_ = false;
    bool warm_on_ = false;
    bool warm_pending_ = false;
    int warm_B_ = 0;
    std::vector<int> warm_R_;
    std::vector<int> warm_parent_;

    bool force_simt_ = false;
    bool tc_ = false;  // tensor-core schedule for the current chunk
    bool tc_eligible() const;
    void forward_start_tc(StartPlan& sp, int B, int nspec, bool save, bool alpha, cudaStream_t s);

    // Adam step of the current alpha iteration (fused into the adjoint).
    const int* adam_active_ = nullptr;
    float adam_step_ = 0.f;
    float adam_bc2_sqrt_ = 1.f;

    // Contraction-kernel timing (lb200_set_profiling).
    bool profile_ = false;
    std::vector<cudaEvent_t> ev_pool_;
    size_t ev_used_ = 0;
    double contraction_flops_ = 0.0;
    int64_t contraction_launches_ = 0;
    void prof_begin(cudaStream_t s);
    void prof_end(cudaStream_t s, double flops);
    double prof_collect();
};

}  // namespace lb200
