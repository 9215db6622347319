// conv_kernels.cuh -- convolution layers of the backward substitution
// (BoundedConvNode), kept as windows over HWC feature maps.
//
// Feature maps of conv layers are stored HWC (channels fastest) per box; a
// flat index (y * W + x) * C + c.  Luna flattens (C, H, W) maps in CHW
// order: the engine permutes at its edges (input boxes, the columns of a
// Linear after a Flatten, row order of a start, intermediate-bound dumps).
//
// A row of a conv start (one unstable neuron at pixel (y0, x0) of the start
// map) is nonzero only on a window of each map below it: the receptive field,
// growing by (w - 1) * stride + kernel per conv.  Such rows are stored as
// dense windows [wh, ww, C] whose top-left pixel on the map is
//   origin = (mul_y * y0 + off_y, mul_x * x0 + off_x);
// window pixels that fall outside the map hold exact zeros.  This is Luna's
// patches mode (Patches.h, BoundedConvNode.cpp:556-709) without the unfold
// copies.  Rows of the output start and of Linear starts cover whole maps
// ("full" windows: origin 0, window = map).
#pragma once

#include "kernels.cuh"

namespace lb200 {

struct WinGeo {
    int C = 1, H = 1, W = 1;       // map at this level (HWC)
    int wh = 1, ww = 1;            // window rows / columns
    int mul_y = 0, mul_x = 0;      // origin = mul * start pixel + off
    int off_y = 0, off_x = 0;
    int st_C = 1, st_W = 1;        // start map channels / width (decode of row_id)
    int full = 1;                  // window == map at origin 0
    __host__ __device__ int size() const { return wh * ww * C; }
};

// Concretisation forms (CROWNAnalysis.cpp:1164-1224 for a matrix A,
// :791-848 with Patches::matmul for patches).
enum : int { CONC_DENSE = 0, CONC_PATCHES = 1 };

// One conv layer seen from a start: transposed convolution of the A window
// at the layer's output (in_h x in_w x Co) into the window at its input
// (out_h x out_w x Ci):
//   out[v, ci] = sum over co and taps k with v + c = q s + k, 0 <= q < in,
//                of A[q, co] W[co, ci, k]
// (BoundedConvNode::boundOneSide, conv_transpose2d, :448-491 / :596-618).
// c = 0 for windows (the whole transposed-conv output) and c = padding for
// full maps (the output cropped to the map).
struct ConvStep {
    int Co = 0, Ci = 0, kh = 0, kw = 0, sh = 1, sw = 1;
    int in_h = 0, in_w = 0, out_h = 0, out_w = 0;
    int cy = 0, cx = 0;
    const float* Wk = nullptr;  // [kh][kw][Co][Ci]
    const float* Wc = nullptr;  // [Co][kh][kw][Ci]
};

// ---- IBP ------------------------------------------------------------------
// W+/W- convolution of HWC interval maps (BoundedConvNode.cpp:864-943); the
// input is clamped at 0 first when it is a ReLU output.
void launch_ibp_conv(const float* Wc, const float* b, const float* in_l, const float* in_u, float* out_l,
                     float* out_u, int B, int Ci, int Hi, int Wi, int Co, int Ho, int Wo, int kh, int kw,
                     int sh, int sw, int ph, int pw, bool relu_in, cudaStream_t s);

// Per-box CHW <-> HWC permutation of [B, C*H*W].
void launch_chw_to_hwc(const float* src, float* dst, int B, int C, int H, int W, cudaStream_t s);

// Row maps of a conv start: unstable neurons in Luna's CHW order, row_id =
// HWC index.  Same warp-per-box compaction as launch_fill_rows.
void launch_fill_rows_chw(const float* l, const float* u, int B, int C, int H, int W, const int* box_off,
                          int* row_box, int* row_id, cudaStream_t s);

// ---- forward (backward-substitution) steps ------------------------------
// Start step of a conv start: the row of neuron (y0, x0, co) is the window
// W[co] (kh x kw x Ci) at the level below (identity patches through the
// start conv, BoundedConvNode.cpp:620-656), bias0 = b[co]; then the ReLU
// relaxation below (masked outside the map) -> Q, bias partial.
struct ConvStartStep {
    RowMap rows;
    int M = 0;
    const float* Wc = nullptr;     // [Co][kh][kw][Ci] of the start conv
    const float* bW = nullptr;     // [Co]
    WinGeo g;                      // window at the level below the start
    WinGeo wg;                     // when g is a whole map: the weight window's placement
    ReluParams rp;                 // ReLU below (rp.n = map size)
    const float* alpha = nullptr;  // [2R, g.size()] or null
    const float* b_next = nullptr; // [C] bias of the layer producing the map below
    float* P_save = nullptr;       // [M, g.size()] or null
    float* Q = nullptr;            // [M, g.size()]
    float* bias_acc = nullptr;     // [M]
};
void launch_conv_start_step(const ConvStartStep& st, cudaStream_t s);

// Transposed-conv step with the ReLU relaxation of the level below in the
// epilogue (Q = relax(P), masked outside the map), or with the input
// concretisation (dense or patches form).  Per-row partial sums go to
// partial[chunk * M + r], chunk = 256-element chunk of the output window;
// conv_chunks() gives their number.
struct ConvRelaxEpi {
    RowMap rows;
    WinGeo g;                      // output window geometry
    ReluParams rp;
    const float* alpha = nullptr;
    const float* b_next = nullptr; // [C]
    float* P_save = nullptr;
    float* Q = nullptr;
    const float* addend = nullptr; // [M, g.size()] or null: skip edges' A, added to P before the relaxation
};
struct ConvConcEpi {
    RowMap rows;
    WinGeo g;
    int form = CONC_DENSE;
    const float* xl = nullptr;     // [B, n0] HWC
    const float* xu = nullptr;
    uint8_t* sign = nullptr;       // [M, g.size()] or null
};
int conv_chunks(const WinGeo& out);
void launch_convT_relax(const float* A, const ConvStep& cs, int M, const ConvRelaxEpi& e, float* partial,
                        cudaStream_t s);
void launch_convT_conc(const float* A, const ConvStep& cs, int M, const ConvConcEpi& e, float* partial,
                       cudaStream_t s);

// Register-blocked forms of the two SIMT conv steps for layers with few
// channels on the output side of the step (8, 16 or 32): one thread per
// window pixel keeps all of that pixel's channels in registers, the layer's
// weights sit in shared memory (at most 48 KB), and every element is summed
// in the same order as launch_convT_relax / launch_conv_adj_qbar (identical
// A and Qbar; the per-row bias partials are grouped differently).  The
// forward step writes one partial per (row, 256-pixel chunk):
// convT_rb_chunks() of them.
bool convT_rb_ok(const ConvStep& cs);
int convT_rb_chunks(const WinGeo& out);
void launch_convT_relax_rb(const float* A, const ConvStep& cs, int M, const ConvRelaxEpi& e, float* partial,
                           cudaStream_t s);
bool conv_adj_rb_ok(const ConvStep& cs);
void launch_conv_adj_qbar_rb(const float* Pbar, const ConvStep& cs, int M, const float* gseed, const float* b,
                             float* Qbar, cudaStream_t s);

// ReLU relaxation of a level from its raw A window P (stored by a tensor-core
// step): Q = relax(P) masked outside the map, bias partials (intercepts +
// Q . b_next per row) into partial[chunk * M + r], one chunk per 1024
// elements of a row (relax_window_chunks).  e.P_save is not used; with
// e.addend, P + addend is written back to P first.
int relax_window_chunks(const WinGeo& g);
void launch_relax_window(float* P, const ConvRelaxEpi& e, int M, float* partial, cudaStream_t s);

// ---- adjoint --------------------------------------------------------------
// d loss / d A at the input window from the concretisation signs: dense form
// (bit0 A>=0, bit1 A<=0) g (xa [bit0] + xb [bit1]); patches form (bit0 A>0,
// bit1 A<0) g c -/+ g d sgn(A) (autograd of A c -/+ |A| d).  Zero outside
// the map.
void launch_win_input_seed(const RowMap& rows, int M, const WinGeo& g, int form, const uint8_t* sign,
                           const float* gseed, const float* xl, const float* xu, float* Pbar0,
                           cudaStream_t s);
// Adjoint of a transposed-conv step: Qbar[q, co] = sum over ci, taps of
// Pbar[v = q s + k - c, ci] W[co, ci, k] + g b[co] (a strided correlation
// of the window below with W).
void launch_conv_adj_qbar(const float* Pbar, const ConvStep& cs, int M, const float* gseed,
                          const float* b, float* Qbar, cudaStream_t s);
// Relaxation adjoint on windows (same rules as launch_relax_adjoint):
// Pbar, the fused projected-Adam step on alpha, and d loss / d (k_up, b_up)
// added into kbar / bbar [B, n] per neuron with atomics.
void launch_relax_adjoint_win(const EpiRelaxAdj& e, const WinGeo& g, const float* Qbar, int M,
                              cudaStream_t s);
// First conv layer with few channels (kh = kw = 3, Ci = 3, Co <= 32, stride
// 1): its transposed-conv step fused with the input concretisation, and its
// adjoint fused with the input seed.  One CTA per row, one output pixel per
// warp iteration, lane = output channel of the conv (its 27 weights in
// registers).  The concretisation writes one partial per row (slot 0).
bool first_conv_fast(const ConvStep& cs);
void launch_first_convT_conc(const float* A, const ConvStep& cs, int M, const ConvConcEpi& e, float* partial,
                             cudaStream_t s);
void launch_first_conv_adj(const RowMap& rows, int M, const WinGeo& g0, int form, const uint8_t* sign,
                           const float* gseed, const float* xl, const float* xu, const ConvStep& cs,
                           const float* b, float* Qbar, cudaStream_t s);

// ---- transposed-conv layers (BoundedConvTransposeNode) -------------------
// Geometry of a ConvTranspose2d layer: in (Ci, Hi, Wi) -> out (Co, Ho, Wo),
// Ho = (Hi - 1) s - 2 p + kh; out[v] gets in[q] W[ci, co, k] for v = q s - p + k.
// Rows through such a layer are whole maps.
struct ConvTStep {
    int Ci = 0, Co = 0, kh = 0, kw = 0, sh = 1, sw = 1, ph = 0, pw = 0;
    int Hi = 0, Wi = 0, Ho = 0, Wo = 0;
    const float* Wg = nullptr;  // [Ci][kh][kw][Co]
    const float* Wa = nullptr;  // [kh][kw][Co][Ci]
};
// Centre / radius IBP (BoundedConvTransposeNode.cpp:466-488): c = convT(mid)
// + b, d = convT(diff, |W|), [c - d, c + d]; inputs clamped at 0 first when
// they are a ReLU output.
void launch_ibp_convt(const ConvTStep& ct, const float* b, const float* in_l, const float* in_u, float* out_l,
                      float* out_u, int B, bool relu_in, cudaStream_t s);
// Back-substitution through the layer (a strided correlation,
// BoundedConvTransposeNode.cpp:250-280): P_in[q, ci] = sum_{k, co}
// A_out[q s - p + k, co] W[ci, co, k], with the ReLU relaxation of the level
// below in the epilogue (whole maps; chunk partials as launch_convT_relax).
void launch_convt_back_relax(const float* A, const ConvTStep& ct, int M, const ConvRelaxEpi& e, float* partial,
                             cudaStream_t s);
// Register-blocked forms of the two steps (whole maps; the same per-element
// summation order): one thread per pixel and 16 (back-substitution) or 8
// (adjoint) channels, the weights of that channel group in shared memory.
// The back-substitution writes convt_rb_chunks() partials per row.
bool convt_rb_ok(const ConvTStep& ct);
int convt_rb_chunks(const ConvTStep& ct);
void launch_convt_back_relax_rb(const float* A, const ConvTStep& ct, int M, const ConvRelaxEpi& e, float* partial,
                                cudaStream_t s);
bool convt_adj_rb_ok(const ConvTStep& ct);
void launch_convt_adj_qbar_rb(const float* Pbar, const ConvTStep& ct, int M, float* Qbar, cudaStream_t s);
// Start step of a ConvTranspose start: the one-hot row at output neuron
// (v0, co0) through the layer is W[:, co0, k] at the q with q s - p + k = v0;
// the layer's bias does not enter (flat A, see launch_convt_back_relax).
void launch_convt_start_step(const ConvStartStep& st, const ConvTStep& ct, cudaStream_t s);
// Adjoint of the back-substitution step: Qbar[v, co] = sum P_in[q, ci]
// W[ci, co, k] over v = q s - p + k (a transposed conv; no bias term).
void launch_convt_adj_qbar(const float* Pbar, const ConvTStep& ct, int M, float* Qbar, cudaStream_t s);

// ---- residual joins (BoundedAddNode) ---------------------------------------
// A skip edge carries the A at an Add (level i) to the ReLU output of level j
// that feeds it, directly or through a conv; there it joins the A of the
// main path before level j's relaxation (CROWNAnalysis::addA, :1248-1355;
// BoundedAddNode::boundBackward, :167-279).  In window coordinates the skip
// conv maps Q_i pixel q to S_j pixel v = q s + k - c (identity: v = q - c).
struct SkipStep {
    WinGeo gi, go;              // windows at level i (Q) and level j (S)
    int Co = 0, Ci = 0;         // channels of level i / level j (equal for identity)
    int kh = 1, kw = 1, sh = 1, sw = 1;
    int cy = 0, cx = 0;
    const float* Wk = nullptr;  // [kh][kw][Co][Ci]; null: identity
    const float* Wc = nullptr;  // [Co][kh][kw][Ci]; null: identity
};
// S[r, v] += (skip^T Q)[r, v] over the window at level j; Q == null stands
// for the one-hot rows of a start at level i (the start's own neuron).
void launch_skip_back(const SkipStep& k, const RowMap& rows, int M, const float* Q, float* S, cudaStream_t s);
// Adjoint: Qbar[r, q] += (skip Pbar)[r, q], Pbar in the window layout of
// level j or phase-split as `ps` describes.
void launch_skip_adj(const SkipStep& k, const RowMap& rows, int M, const float* Pbar, const PhaseSplit& ps,
                     float* Qbar, cudaStream_t s);

// dst[i] += (float)src[i], src[i] = 0 for i < n (folds the double scratch of
// launch_relax_adjoint_win into kbar / bbar).
void launch_fold_double(double* src_k, double* src_b, float* dst_k, float* dst_b, int64_t n, cudaStream_t s);

// alpha[p][r][j] = init_slope[box, neuron(r, j)] (0 outside the map).
void launch_alpha_init_win(const RowMap& rows, const WinGeo& g, const float* init_slope, int n,
                           float* alpha, cudaStream_t s);

}  // namespace lb200
