// kernels.cuh -- device kernels of the luna_b200 engine and their launchers.
//
// Data layout in HBM (B boxes, one backward start with R rows per side):
//   per-box vectors          [B, n]      row-major, box-major
//   A matrices of a start    [2R, n]     rows 0..R-1 lower side (lA),
//                                        rows R..2R-1 upper side (uA)
//   alpha of (relu m, start) [2R, n_m]   same row order as A; only the
//                                        neurons flagged RF_USE_ALPHA are read
//   row maps                 row_box[R], row_id[R]: rows sorted by box, then
//                                        by neuron (intermediate start) or
//                                        spec index (output start)
#pragma once

#include "common.cuh"

namespace lb200 {

struct RowMap {
    const int* row_box = nullptr;  // [R]
    const int* row_id = nullptr;   // [R] neuron id (intermediate) or spec index (output)
    const int* box_off = nullptr;  // [B+1] first row of each box
    int R = 0;
};

struct ReluParams {
    const float* slope_lo = nullptr;  // [B, n] lower slope when the alpha tensor is not read
    const float* k_up = nullptr;      // [B, n] upper slope
    const float* b_up = nullptr;      // [B, n] upper intercept
    const uint8_t* flags = nullptr;   // [B, n] RF_* bits
    const float* b_lo = nullptr;      // [B, n] lower intercept (Sigmoid); null: 0 (ReLU)
    int n = 0;
};

// ---- IBP ----------------------------------------------------------------
// out = W+ l + W- u + b, W+ u + W- l + b for every box; the input bounds are
// clamped at 0 first when `relu_in` (the ReLU node's IBP).
void launch_ibp_linear(const float* W, const float* b, const float* in_l, const float* in_u,
                       float* out_l, float* out_u, int B, int n_in, int n_out, bool relu_in,
                       cudaStream_t s);
// Interval sum of an Add (BoundedAddNode::computeIntervalBoundPropagation,
// :281-304): out += in over n entries; in clamped at 0 first when it is a
// ReLU output.
void launch_add_bounds(float* out_l, float* out_u, const float* in_l, const float* in_u, int64_t n, bool relu_in,
                       cudaStream_t s);

// ---- row maps ------------------------------------------------------------
// counts[b] = #{i : l[b,i] < 0 < u[b,i]}
void launch_count_unstable(const float* l, const float* u, int B, int n, int* counts, cudaStream_t s);
// box_off = exclusive scan of counts (B+1 entries), computed on the device.
void launch_scan_counts(const int* counts, int B, int* box_off, cudaStream_t s);
void launch_fill_rows(const float* l, const float* u, int B, int n, const int* box_off,
                      int* row_box, int* row_id, cudaStream_t s);
void launch_fill_spec_rows(int B, int nspec, int* row_box, int* row_id, int* box_off, cudaStream_t s);

// ---- relaxation parameters ----------------------------------------------
// From the current bounds of a ReLU's input compute slope_lo / k_up / b_up /
// flags for every (box, neuron).  alpha_mode selects the optimisation-stage
// rules (BoundedReLUNode::_maskAlpha) for boxes whose box_has_aset is set.
// When `create` is set the alpha-creation mask and initial slope are taken
// from these bounds (aset, init_slope, box_has_aset are written).
void launch_relu_params(const float* l, const float* u, int B, int n, bool alpha_mode, bool create,
                        uint8_t* aset, float* init_slope, int* box_has_aset, float* slope_lo,
                        float* k_up, float* b_up, uint8_t* flags, cudaStream_t s);
// alpha[p][r][j] = init_slope[row_box[r], j] for both sides.
void launch_alpha_init(const RowMap& rows, const float* init_slope, int n, float* alpha, cudaStream_t s);

// ---- backward-substitution steps ------------------------------------------
// Start step: P[r] = spec_row(r) . W (spec_row = one-hot of row_id for an
// intermediate start, C[box, row_id] for the output start), bias0[r] =
// spec_row . b; then the ReLU relaxation below (when rp.n > 0) producing
// Q = relax(P) and the bias partial (relax intercepts + Q . b_next).
// Writes P_save (may be null), Q, and bias_acc[r] = bias0 + partial.
struct StartStep {
    RowMap rows;
    int M = 0;              // rows in this launch (2R, or R for lower side only)
    const float* W = nullptr;  // [n_spec_dim, n] weight of the start's Linear
    const float* bW = nullptr; // [n_spec_dim] its bias
    int spec_dim = 0;          // rows of W (output features of the Linear)
    const float* C = nullptr;  // output start: [Cb, nspec, spec_dim]; null = one-hot
    int c_per_box = 0;         // 1 if C has one matrix per box
    int nspec = 0;
    int n = 0;                 // columns of P (input features of the Linear)
    ReluParams rp;             // rp.n == 0: no ReLU below (P is concretised)
    const float* alpha = nullptr;
    const float* b_next = nullptr;
    float* P_save = nullptr;
    float* Q = nullptr;
    float* bias_acc = nullptr;
};
void launch_start_step(const StartStep& st, cudaStream_t s);

// GEMM P = A . B (A [M,K] row-major, B [K,N] row-major) with one of three
// fused epilogues.  Each writes a per-row partial sum into
// partial[tile_n * M + r] (tile_n = column tile index), so that the row
// totals are reduced deterministically by launch_sum_partials.
struct EpiRelaxFwd {
    RowMap rows;
    ReluParams rp;
    const float* alpha = nullptr;   // [2R, N] or null
    const float* b_next = nullptr;  // [N] bias of the next Linear below, or null
    float* P_save = nullptr;        // [M, N] or null
    float* Q = nullptr;             // [M, N]
};
struct EpiConcretize {
    RowMap rows;
    const float* xl = nullptr;      // [B, N]
    const float* xu = nullptr;
    uint8_t* sign = nullptr;        // [M, N] or null: bit0 P>=0, bit1 P<=0
};
// Layout of Pbar when the layer above it takes its adjoint on tensor cores
// as a strided correlation: the window (out_h x out_w x C, row-major HWC)
// split into s*s phase planes of nty x ntx pixels, window pixel v sitting in
// plane ((v + c) mod s) at t = (v + c) div s - tlo.  Slots that no window
// pixel maps to stay zero (the caller clears the rows first).
struct PhaseSplit {
    int s = 0;  // 0: Pbar keeps the window layout
    int C = 0, out_w = 0, cy = 0, cx = 0, tlo_y = 0, tlo_x = 0, nty = 0, ntx = 0;
    int64_t row_stride = 0;  // s * s * nty * ntx * C
};
#ifdef __CUDACC__
__device__ __forceinline__ int64_t phase_dst(const PhaseSplit& ps, int64_t r, int j) {
    const int c = j % ps.C, pix = j / ps.C;
    const int vy = pix / ps.out_w + ps.cy, vx = pix - (pix / ps.out_w) * ps.out_w + ps.cx;
    const int plane = (vy % ps.s) * ps.s + vx % ps.s;
    const int ty = vy / ps.s - ps.tlo_y, tx = vx / ps.s - ps.tlo_x;
    return r * ps.row_stride + (((int64_t)plane * ps.nty + ty) * ps.ntx + tx) * ps.C + c;
}
#endif

struct EpiRelaxAdj {
    PhaseSplit ps;  // launch_relax_adjoint / launch_relax_adjoint_win only
    RowMap rows;
    ReluParams rp;
    const float* gseed = nullptr;   // [M] bias adjoint of each row
    const float* b_lin = nullptr;   // [N] bias of the Linear whose W^T is the B operand
    const float* P_saved = nullptr; // [M, N] pre-relaxation A saved by the forward pass
    float* alpha = nullptr;         // [2R, N] or null
    float* Pbar = nullptr;          // [M, N] or null
    float* alpha_grad = nullptr;    // [2R, N] or null (gradient output when Adam is not fused)
    // Fused projected Adam: when adam_m != null, each alpha entry of the rows
    // of an active box takes its Adam step in place right after its gradient
    // is formed (each alpha of a start gets its gradient from exactly one
    // element of this epilogue), and no gradient buffer is written.
    float* adam_m = nullptr;        // [2R, N]
    float* adam_v = nullptr;
    const int* active = nullptr;    // [B]
    float adam_step = 0.f;          // lr / bias_correction1
    float adam_bc2_sqrt = 1.f;      // sqrt(bias_correction2)
    // Per-(row group, virtual box) partial sums of d loss / d k_up and
    // d loss / d b_up, reduced in a fixed order by launch_reduce_relax_grad.
    // The virtual box of row r is box + side * B; slot = r / group + virtual
    // box is unique because rows are sorted by virtual box.
    float* kslot = nullptr;         // [(ceil(M/group) + 2B), N]
    float* bslot = nullptr;
    // Sigmoid levels (rp.b_lo set): also d loss / d slope_lo and d loss /
    // d b_lo, for every neuron.
    float* sslot = nullptr;
    float* blslot = nullptr;
    int B = 0;
    // Direct accumulators [B, N] (launch_relax_adjoint).
    float* kbar = nullptr;
    float* bbar = nullptr;
    // Double-precision scratch [B, N] of launch_relax_adjoint_win: its
    // atomics accumulate here (rounding error far below fp32 resolution, so
    // the fp32 totals do not depend on the atomic order) and
    // launch_fold_double adds the totals into kbar / bbar.
    double* kbar_d = nullptr;
    double* bbar_d = nullptr;
    // launch_relax_adjoint: when set, the pre-relaxation A of row r is the
    // weight row gather_W[row_id[r]] (ReLU directly below a one-hot start)
    // and P_saved is not read.
    const float* gather_W = nullptr;
    // First adjoint step on the tensor-core path: the A operand (d loss / d A
    // at the input) is generated in the kernel from the concretisation signs
    // instead of being read from memory (see launch_adj_input_seed).
    const uint8_t* seed_sign = nullptr;  // [M, K]
    const float* seed_xl = nullptr;      // [B, K]
    const float* seed_xu = nullptr;
};
void launch_gemm_relax_fwd(const float* A, const float* Bm, int M, int N, int K,
                           const EpiRelaxFwd& e, float* partial, cudaStream_t s);
void launch_gemm_concretize(const float* A, const float* Bm, int M, int N, int K,
                            const EpiConcretize& e, float* partial, cudaStream_t s);
void launch_gemm_relax_adj(const float* A, const float* Bm, int M, int N, int K,
                           const EpiRelaxAdj& e, float* partial, cudaStream_t s);
int gemm_tiles_n(int N);

// Adjoint contraction whose epilogue only adds g[r] b_lin[c] and stores
// Qbar = A . B + g b_lin (tensor-core path; the relaxation adjoint then runs
// in launch_relax_adjoint).  Uses the seed_* fields of `e` for the first step.
struct EpiStoreQbar {
    const float* gseed = nullptr;   // [M]
    const float* b_lin = nullptr;   // [N]
    float* Qbar = nullptr;          // [M, N]
    RowMap rows;                    // seed generation only
    const uint8_t* seed_sign = nullptr;
    const float* seed_xl = nullptr;
    const float* seed_xu = nullptr;
};

// Relaxation adjoint of ReLU m for the rows of one start, from Qbar: writes
// Pbar (may be null), takes the fused projected-Adam step of alpha (rows of
// active boxes), and adds this start's d loss / d k_up and d loss / d b_up
// into kbar / bbar [B, n] in a fixed order (one CTA per box and 32 columns,
// both sides).  M = 2R, or R for the lower side only.
void launch_relax_adjoint(const EpiRelaxAdj& e, const float* Qbar, int M, int n, cudaStream_t s);

// kbar[b, c] += sum of the slots of virtual boxes b and B + b (rows < M), in
// row order, for the slot layout of EpiRelaxAdj with `group`-row groups
// (8 for the SIMT kernel, 32 for the tensor-core kernel).
void launch_reduce_relax_grad(const RowMap& rows, int M, int B, int N, int group, const float* kslot,
                              const float* bslot, float* kbar, float* bbar, cudaStream_t s);

// ---- Sigmoid (BoundedSigmoidNode) -------------------------------------------
// Relaxation lw x + lb <= sigmoid(x) <= uw x + ub on [l, u] per neuron
// (boundRelaxImpl, BoundedSigmoidNode.cpp:282-338): secants where valid, the
// midpoint tangent on the convex / concave side, and across 0 the tangent
// points of Luna's tables (:75-151, entry max(0, int(b / 0.01)) + 1 of the
// bound, :162-186), each entry found here by the same doubling and 100-step
// fp32 bisection.  Writes slope_lo = lw, b_lo = lb, k_up = uw, b_up = ub and
// flags RF_UNSTABLE (every neuron passes its parameter adjoints on).
void launch_sigmoid_params(const float* l, const float* u, int B, int n, float* lw, float* lb, float* uw, float* ub,
                           uint8_t* flags, cudaStream_t s);
// d loss / d (l, u) of start row r's neuron from d loss / d (lw, lb, uw, ub)
// (sbar, blbar, kbar, bbar), by the derivatives of the secant and midpoint
// lines (the table tangents do not depend on l, u): g[r] and g[R + r].
void launch_sigmoid_bound_grad(const RowMap& rows, const float* cur_l, const float* cur_u, const float* sbar,
                               const float* blbar, const float* kbar, const float* bbar, int n, float* g,
                               cudaStream_t s);
// Sigmoid output bounds [sigmoid(l), sigmoid(u)] (monotone, :248-272).
void launch_sigmoid_bounds(const float* l, const float* u, float* ol, float* ou, int64_t n, cudaStream_t s);
int relax_grad_slots(int M, int B, int group);

// out[r] = base[r] + sum_t partial[t * M + r] for t in [0, ntiles).
void launch_sum_partials(const float* base, const float* partial, int ntiles, int M, float* out,
                         cudaStream_t s);

// ---- start finalisation ---------------------------------------------------
// Intermediate start: the CROWN bound of row r is val[r] (lower) and
// val[R + r] (upper).  Write into cur_l / cur_u [B, n] at (box, neuron),
// applying the STE clamp against ref (when ref_l != null):
// lower = (max(ref, c) - c) + c, upper = c - (c - min(ref, c)).
void launch_scatter_start(const RowMap& rows, const float* val, const float* ref_l,
                          const float* ref_u, int n, float* cur_l, float* cur_u, cudaStream_t s);
// Output start: lb[b, j] = val[r], ub[b, j] = val[R + r] (when has_upper).
void launch_scatter_output(const RowMap& rows, const float* val, int nspec, bool has_upper,
                           float* lb, float* ub, cudaStream_t s);

// ---- alpha-CROWN control ----------------------------------------------------
struct BoxControl {
    float* best = nullptr;          // [B, nspec] best lower bound so far
    float* best_loss = nullptr;     // [B] |loss| at the last reset
    int* patience = nullptr;        // [B]
    int* active = nullptr;          // [B] 1 while the box is optimising
    int* has_best = nullptr;        // [B]
    int* save = nullptr;            // [B] set when this iteration saves alpha/bounds
    uint8_t* improved = nullptr;    // [B, nspec]
    int* first_save = nullptr;      // [B] 1 until the first alpha save
    // STOP_ALPHA_ON_VERIFIED with thresholds (thr != null): a box whose
    // current lower bounds verify the specification stops at once.
    const float* thr = nullptr;     // [nspec]
    const int32_t* branch = nullptr; // [nspec] OR branch of each row (n_branches > 0)
    int n_branches = 0;
    int* n_active = nullptr;        // [1] boxes still optimising after this iteration
};
// One iteration's bookkeeping (AlphaCROWNAnalysis.cpp:394-472) for every
// active box.  `cur` is the bound being maximised [B, nspec]: the current
// lower bound, or the negated upper bound when the upper side is optimised
// (best = min, improvement = decrease and loss = sum of ub are then the same
// arithmetic).  `verify` [B, nspec] (or null: `cur`) holds the lower bounds
// that STOP_ALPHA_ON_VERIFIED checks (isSpecVerified reads lower bounds on
// either side, AlphaCROWNAnalysis.cpp:396-407).
void launch_alpha_control(const BoxControl& c, const float* cur, const float* verify, int B, int nspec, int iter,
                          int save_after, int patience_limit, bool has_loss, cudaStream_t s);
// STOP_CROWN_ON_VERIFIED (TorchModel.cpp:816-834): done[b] = the box's CROWN
// lower bounds lb [B, nspec] verify the specification; active[b] = !done[b];
// *n_done counts the done boxes (set to zero first by the caller).
void launch_crown_verified(const float* lb, const float* thr, const int32_t* branch, int n_branches, int B,
                           int nspec, int* done, int* active, int* n_done, cudaStream_t s);
// lb, ub [B, nspec] = crown_lb, crown_ub for the boxes with done.
void launch_take_verified(const int* done, const float* crown_lb, const float* crown_ub, int B, int nspec,
                          float* lb, float* ub, cudaStream_t s);
// best_l = max(best_l, cur_l), best_u = min(best_u, cur_u) for boxes with save.
void launch_snapshot(const int* save, const float* cur_l, const float* cur_u, int B, int n,
                     float* best_l, float* best_u, cudaStream_t s);
// Copy alpha rows into best_alpha for boxes with save: every row the first
// time, then the rows whose index within the box is an improved spec index.
void launch_best_alpha(const RowMap& rows, const int* save, const int* first_save,
                       const uint8_t* improved, int nspec, int n, const float* alpha,
                       float* best_alpha, cudaStream_t s);
// After the first save: only rows with index < nspec inside their box can be
// copied, so launch over B x nspec rows per side instead of all rows.
void launch_best_alpha_rows(const RowMap& rows, int B, const int* save, const uint8_t* improved,
                            int nspec, int n, const float* alpha, float* best_alpha, cudaStream_t s);
void launch_clear_first_save(const int* save, int* first_save, int B, cudaStream_t s);
// Projected Adam (torch::optim::Adam + clamp to [0,1]) on the rows of active boxes.
void launch_adam(const RowMap& rows, const int* active, int n, float* alpha, float* m, float* v,
                 const float* grad, float step_size, float bc2_sqrt, cudaStream_t s);
// lb = max(final, best) for every box.
void launch_max_best(const float* best, const int* has_best, int total, int nspec, float* lb,
                     cudaStream_t s);

// ---- adjoint helpers --------------------------------------------------------
// Pbar0[r, j] = g[r] * (x_a[b, j] if P >= 0) + g[r] * (x_b[b, j] if P <= 0),
// x_a/x_b = xl/xu for the lower side and xu/xl for the upper side.
void launch_adj_input_seed(const RowMap& rows, int M, const uint8_t* sign, const float* g,
                           const float* xl, const float* xu, int n0, float* Pbar0, cudaStream_t s);
// Chain rule from (kbar, bbar) of a ReLU to the bounds of its input, written
// as the seeds of the rows of that input's start: g[r] (lower) and g[R + r].
void launch_bound_grad(const RowMap& rows, const float* cur_l, const float* cur_u,
                       const uint8_t* flags, const float* kbar, const float* bbar, int n,
                       float* g, cudaStream_t s);
// Output-start seed: g[r] = -1 for rows of active boxes (loss = -sum lb), 0 else.
void launch_output_seed(const RowMap& rows, const int* active, float* g, cudaStream_t s);
// Output-start seed for the upper side [2R]: 0 on the lower rows, +1 on the
// upper rows of active boxes (loss = sum ub, AlphaCROWNAnalysis::computeLoss).
void launch_output_seed_upper(const RowMap& rows, const int* active, float* g, cudaStream_t s);
// out[i] = -in[i].
void launch_negate(const float* in, float* out, int64_t n, cudaStream_t s);

// alpha = best_alpha on the rows of boxes that saved at least once
// (AlphaCROWNAnalysis::restoreBestAlphas).
void launch_restore_alpha(const RowMap& rows, const int* first_save, int n, const float* best_alpha,
                          float* alpha, cudaStream_t s, const int* keep_current = nullptr);
// ---- warm start (TorchModel::loadState / seedAlphas) --------------------------
// seed[b] = 1 when box b has a parent (parent[b] >= 0) whose start had as many
// rows as box b's (AlphaCROWNAnalysis::ensureAlphaFor reuses a seeded alpha
// only when its specification count matches).
void launch_warm_seed(const int* box_off, const int* prev_box_off, const int* parent, int B, int* seed,
                      cudaStream_t s);
// Seeded boxes' alpha rows (both sides) copied from the parent's rows by
// position within the box.
void launch_warm_alpha(const RowMap& rows, const int* seed, const int* parent, const int* prev_box_off, int prev_R,
                       int n, const float* prev_alpha, float* alpha, cudaStream_t s);
// The creation set of one (ReLU, start) per box: the parent's for seeded
// boxes, the box's own otherwise; has[b] = it is non-empty.
void launch_warm_aset(const int* seed, const int* parent, int B, int n, const uint8_t* prev_aset,
                      const uint8_t* aset, uint8_t* out, int* has, cudaStream_t s);
// IBP of the specification: lb = C+ l + C- u, ub = C+ u + C- l per box.
void launch_ibp_spec(const float* C, int c_per_box, const float* l, const float* u, int B, int nspec,
                     int nout, float* lb, float* ub, cudaStream_t s);

// Sub on the input node (BoundedSubNode's interval forward): per box,
// [xl - c, xu - c], or [c - xu, c - xl] when neg (constant first).
void launch_input_sub(const float* c, bool neg, const float* xl, const float* xu, float* ol, float* ou, int B, int n,
                      cudaStream_t s);

// Fill / copy helpers.
void launch_fill_f32(float* p, float v, int64_t n, cudaStream_t s);
void launch_expand_spec(const float* C, int c_per_box, int B, int nspec, int nout, float* out,
                        cudaStream_t s);

}  // namespace lb200
