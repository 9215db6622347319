// tc_conv.cuh -- sm_100a tensor-core (tcgen05 + TMEM + TMA, 3xTF32) conv
// steps of the backward substitution, weights-stationary implicit GEMM.
//
//   D[m, n] = sum_k Wmat[m, k] X[n, k]
//
// m runs over weight rows (the MMA's M = 128 per tile), n over a box of
// output pixels of up to BR rows x BY x BX pixels (the MMA's N), and k over
// K blocks of 32 channels, each block reading the data window shifted by one
// tap (a TMA box load of the 5-D data tensor (C, X, Y, P, R) with zero fill
// outside it).
//
// Transposed-conv step (forward, A through a conv layer): the s*s output
// phases are stacked in M (m = phase * Ci + ci), so all phases read the
// same data shift q = t - u per K block: output pixel v = s (t + tlo) +
// phase - c for t in the phase grid, tap k = phase + s u.
// Correlation step (adjoint, Qbar from Pbar): m = co, the data is Pbar
// split into its s*s phase planes so that tap k = phase + s u reads plane
// `phase` at q + u - tlo.
#pragma once

#include "conv_kernels.cuh"

namespace lb200 {

constexpr int TC_CONV_MAX_KB = 96;

struct TcConvTap {
    int plane = 0, dy = 0, dx = 0, c0 = 0;  // data shift and channel block of one K block
};

struct TcConvPlan {
    // Data tensor (C, X, Y, P, R), fp32, row-major with C fastest.  With
    // ds > 1 output pixel (ty, tx) of a K block reads data pixel
    // (ty ds + dy, tx ds + dx): the TMA box traverses X and Y with element
    // stride ds (a strided correlation without a phase-split copy).
    const float* data = nullptr;
    int C = 0, X = 0, Y = 0, P = 1, R = 0;
    int ds = 1;
    // Output pixel grid per row (ny x nx) and its tiling.
    int ny = 0, nx = 0;
    int BR = 1, BY = 1, BX = 1, N = 16;  // N = BR*BY*BX rounded up to 16 (<= 256)
    int nkb = 0;
    TcConvTap kb[TC_CONV_MAX_KB];
    // Weight matrix [m_total, nkb * 32] K-major, tf32 hi / lo.
    const float* w_hi = nullptr;
    const float* w_lo = nullptr;
    int m_total = 0;
};

// Epilogue of a transposed-conv step: D[(phase, ci), t] is the A window of
// the level below at v = s (t + tlo) - c + phase, stored raw into P [rows,
// out_h * out_w * Ci] (the relaxation of that level streams through
// launch_relax_window afterwards).
struct TcConvFwd {
    int s = 1, Ci = 0, cy = 0, cx = 0, tlo_y = 0, tlo_x = 0, out_h = 0, out_w = 0;
    float* P = nullptr;
};
// Epilogue of a correlation step: Qbar[r, (qy * in_w + qx) * Co + co] =
// D[co, q] + g[r] b[co] (D alone when b is null).
struct TcConvQbar {
    int Co = 0, in_w = 0;
    const float* gseed = nullptr;
    const float* b = nullptr;
    float* Qbar = nullptr;
};

// True when the tensor-core conv path handles the step (channel counts
// multiples of 32 on the data side, pixel grid rows <= 256 wide, and no
// wider than 256 / ds data pixels).
bool tc_conv_supported(int data_C, int nx, int ds = 1);
// Tiling of a per-row pixel grid ny x nx over `rows` rows.
void tc_conv_tile(TcConvPlan& p, int rows);
void launch_tc_conv_fwd(const TcConvPlan& p, int rows, const TcConvFwd& e, cudaStream_t s);
void launch_tc_conv_qbar(const TcConvPlan& p, int rows, const TcConvQbar& e, cudaStream_t s);

}  // namespace lb200
