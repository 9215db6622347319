// kernels.cu -- SIMT kernels of the luna_b200 engine (IBP, row maps,
// relaxation parameters, start steps, fp32 GEMM with fused epilogues,
// alpha-CROWN control and the hand-written adjoint).
#include "kernels.cuh"
#include "property.cuh"

#include <algorithm>
#include <cmath>

namespace lb200 {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Path (0 = lower side, 1 = upper side) and per-side row of stacked row r.
__device__ __forceinline__ void split_row(int r, int R, int& p, int& rr) {
    p = r >= R ? 1 : 0;
    rr = r - p * R;
}

}  // namespace

// ============================================================== IBP
__global__ void ibp_linear_kernel(const float* __restrict__ W, const float* __restrict__ bias,
                                  const float* __restrict__ in_l, const float* __restrict__ in_u,
                                  float* __restrict__ out_l, float* __restrict__ out_u, int B,
                                  int n_in, int n_out, bool relu_in) {
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= (int64_t)B * n_out) return;
    const int bx = (int)(warp / n_out), o = (int)(warp % n_out);
    const float* w = W + (size_t)o * n_in;
    const float* l = in_l + (size_t)bx * n_in;
    const float* u = in_u + (size_t)bx * n_in;
    float lp = 0.f, ln = 0.f, up = 0.f, un = 0.f;
    for (int k = lane; k < n_in; k += 32) {
        float wv = w[k], lv = l[k], uv = u[k];
        if (relu_in) {
            lv = fmaxf(lv, 0.f);
            uv = fmaxf(uv, 0.f);
        }
        const float wp = fmaxf(wv, 0.f), wn = fminf(wv, 0.f);
        lp = fmaf(wp, lv, lp);
        ln = fmaf(wn, uv, ln);
        up = fmaf(wp, uv, up);
        un = fmaf(wn, lv, un);
    }
    lp = warp_sum(lp);
    ln = warp_sum(ln);
    up = warp_sum(up);
    un = warp_sum(un);
    if (lane == 0) {
        const float bb = bias ? bias[o] : 0.f;
        out_l[(size_t)bx * n_out + o] = (lp + ln) + bb;
        out_u[(size_t)bx * n_out + o] = (up + un) + bb;
    }
}

void launch_ibp_linear(const float* W, const float* b, const float* in_l, const float* in_u,
                       float* out_l, float* out_u, int B, int n_in, int n_out, bool relu_in,
                       cudaStream_t s) {
    const int64_t threads = (int64_t)B * n_out * 32;
    ibp_linear_kernel<<<ceil_div(threads, 256), 256, 0, s>>>(W, b, in_l, in_u, out_l, out_u, B,
                                                             n_in, n_out, relu_in);
    LB_LAUNCH();
}

// ============================================================== row maps
__global__ void count_unstable_kernel(const float* __restrict__ l, const float* __restrict__ u,
                                      int n, int* __restrict__ counts) {
    const int bx = blockIdx.x;
    int c = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float lv = l[(size_t)bx * n + i], uv = u[(size_t)bx * n + i];
        c += (lv < 0.f && uv > 0.f) ? 1 : 0;
    }
    __shared__ int sh[32];
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
        counts[bx] = t;
    }
}

void launch_count_unstable(const float* l, const float* u, int B, int n, int* counts, cudaStream_t s) {
    count_unstable_kernel<<<B, 256, 0, s>>>(l, u, n, counts);
    LB_LAUNCH();
}

// Exclusive scan of B counts with one block of 1024 threads.
__global__ void scan_counts_kernel(const int* __restrict__ counts, int B, int* __restrict__ off) {
    __shared__ int part[1024];
    const int t = threadIdx.x;
    const int per = (B + 1023) / 1024;
    const int a = t * per, e = min(B, a + per);
    int sum = 0;
    for (int i = a; i < e; ++i) sum += counts[i];
    part[t] = sum;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        int v = (t >= o) ? part[t - o] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    int run = part[t] - sum;
    for (int i = a; i < e; ++i) {
        off[i] = run;
        run += counts[i];
    }
    if (t == 1023) off[B] = part[1023];
}

void launch_scan_counts(const int* counts, int B, int* box_off, cudaStream_t s) {
    scan_counts_kernel<<<1, 1024, 0, s>>>(counts, B, box_off);
    LB_LAUNCH();
}

// One warp per box; unstable neurons in ascending order.
__global__ void fill_rows_kernel(const float* __restrict__ l, const float* __restrict__ u, int B,
                                 int n, const int* __restrict__ off, int* __restrict__ row_box,
                                 int* __restrict__ row_id) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= B) return;
    int base = off[warp];
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        bool un = false;
        if (i < n) {
            const float lv = l[(size_t)warp * n + i], uv = u[(size_t)warp * n + i];
            un = lv < 0.f && uv > 0.f;
        }
        const unsigned m = __ballot_sync(0xffffffffu, un);
        if (un) {
            const int pos = base + __popc(m & ((1u << lane) - 1u));
            row_box[pos] = warp;
            row_id[pos] = i;
        }
        base += __popc(m);
    }
}

void launch_fill_rows(const float* l, const float* u, int B, int n, const int* box_off, int* row_box,
                      int* row_id, cudaStream_t s) {
    fill_rows_kernel<<<ceil_div((int64_t)B * 32, 256), 256, 0, s>>>(l, u, B, n, box_off, row_box,
                                                                    row_id);
    LB_LAUNCH();
}

__global__ void fill_spec_rows_kernel(int B, int nspec, int* row_box, int* row_id, int* box_off) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < (int64_t)B * nspec) {
        row_box[r] = (int)(r / nspec);
        row_id[r] = (int)(r % nspec);
    }
    if (r <= B) box_off[r] = (int)(r * nspec);
}

void launch_fill_spec_rows(int B, int nspec, int* row_box, int* row_id, int* box_off, cudaStream_t s) {
    const int64_t n = (int64_t)B * nspec + 1;
    fill_spec_rows_kernel<<<ceil_div(n, 256), 256, 0, s>>>(B, nspec, row_box, row_id, box_off);
    LB_LAUNCH();
}

// ============================================================== relaxation
// BoundedReLUNode::_reluUpperBound (d = ub_r / (ub_r - lb_r), b = -lb_r d) and
// _computeStandardCROWNLowerBound; _maskAlpha for the optimisation stage.
__global__ void relu_params_kernel(const float* __restrict__ l, const float* __restrict__ u, int B,
                                   int n, bool alpha_mode, bool create, uint8_t* __restrict__ aset,
                                   float* __restrict__ init_slope, const int* __restrict__ has_aset,
                                   float* __restrict__ slope_lo, float* __restrict__ k_up,
                                   float* __restrict__ b_up, uint8_t* __restrict__ flags) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)B * n) return;
    const int bx = (int)(idx / n);
    const float lv = l[idx], uv = u[idx];
    const float lb_r = fminf(lv, 0.f);
    const float ub_r = fmaxf(fmaxf(uv, 0.f), lb_r + 1e-8f);
    const float d = ub_r / (ub_r - lb_r);
    const bool active = lv >= 0.f;
    const bool inactive = uv <= 0.f;
    const bool unstable = lv < 0.f && uv > 0.f;
    const float dlo = active ? 1.f : (unstable ? (d > 0.5f ? 1.f : 0.f) : 0.f);
    if (create) {
        aset[idx] = unstable ? 1 : 0;
        init_slope[idx] = fminf(fmaxf(dlo, 0.f), 1.f);
    }
    if (alpha_mode && has_aset[bx]) {
        k_up[idx] = active ? 1.f : (inactive ? 0.f : d);
        b_up[idx] = (active || inactive) ? 0.f : (-lv) * d;
        slope_lo[idx] = active ? 1.f : 0.f;
        uint8_t f = 0;
        if (aset[idx] && !active) f |= RF_USE_ALPHA;
        if (aset[idx]) f |= RF_ASET;
        if (!active && !inactive) f |= RF_UNSTABLE;
        flags[idx] = f;
    } else {
        k_up[idx] = d;
        b_up[idx] = -lb_r * d;
        slope_lo[idx] = dlo;
        // A box whose alpha for this activation was created empty keeps the
        // CROWN relaxation (BoundedReLUNode::_maskAlpha with no unstable
        // indices); its upper line still depends on the bounds, so in the
        // alpha loop a neuron that has become unstable passes gradient to
        // them.  (With the stabilised intermediate bounds no neuron of such
        // a box can become unstable.)
        flags[idx] = (alpha_mode && unstable) ? RF_UNSTABLE : 0;
    }
}

__global__ void box_any_kernel(const uint8_t* __restrict__ m, int n, int* __restrict__ any) {
    const int bx = blockIdx.x;
    int c = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) c |= m[(size_t)bx * n + i];
    c = __syncthreads_or(c);
    if (threadIdx.x == 0) any[bx] = c ? 1 : 0;
}

void launch_relu_params(const float* l, const float* u, int B, int n, bool alpha_mode, bool create,
                        uint8_t* aset, float* init_slope, int* box_has_aset, float* slope_lo,
                        float* k_up, float* b_up, uint8_t* flags, cudaStream_t s) {
    const int64_t total = (int64_t)B * n;
    if (create) {
        // First pass writes aset; the per-box "any" decides the relaxation mode.
        relu_params_kernel<<<ceil_div(total, 256), 256, 0, s>>>(l, u, B, n, false, true, aset,
                                                                init_slope, box_has_aset, slope_lo,
                                                                k_up, b_up, flags);
        LB_LAUNCH();
        box_any_kernel<<<B, 256, 0, s>>>(aset, n, box_has_aset);
        LB_LAUNCH();
    }
    relu_params_kernel<<<ceil_div(total, 256), 256, 0, s>>>(l, u, B, n, alpha_mode, false, aset,
                                                            init_slope, box_has_aset, slope_lo,
                                                            k_up, b_up, flags);
    LB_LAUNCH();
}

// Row copies [2R, n] <- per-box rows: block (x, y) copies 1024 floats of row y
// (rows beyond gridDim.y in steps of gridDim.y), by float4 when n % 4 == 0.
__device__ __forceinline__ void copy_row(const float* __restrict__ src, float* __restrict__ dst, int n) {
    const int c0 = blockIdx.x * 1024 + threadIdx.x * 4;
    if ((n & 3) == 0) {
        if (c0 < n) *reinterpret_cast<float4*>(dst + c0) = *reinterpret_cast<const float4*>(src + c0);
    } else {
        for (int c = c0; c < min(c0 + 4, n); ++c) dst[c] = src[c];
    }
}

__global__ void alpha_init_kernel(const int* __restrict__ row_box, int R, const float* __restrict__ init,
                                  int n, float* __restrict__ alpha) {
    for (int r2 = blockIdx.y; r2 < 2 * R; r2 += gridDim.y) {
        const int rr = r2 >= R ? r2 - R : r2;
        copy_row(init + (size_t)row_box[rr] * n, alpha + (size_t)r2 * n, n);
    }
}

void launch_alpha_init(const RowMap& rows, const float* init_slope, int n, float* alpha, cudaStream_t s) {
    if (rows.R == 0 || n == 0) return;
    const dim3 grid(ceil_div(n, 1024), std::min(2 * rows.R, 65535));
    alpha_init_kernel<<<grid, 256, 0, s>>>(rows.row_box, rows.R, init_slope, n, alpha);
    LB_LAUNCH();
}

// Forward relaxation of one element.  Lower side: Q = P+ s + P- k, bias
// term P- b; upper side: Q = P+ k + P- s, bias term P+ b
// (BoundedReLUNode.cpp:179-195,268-285).
__device__ __forceinline__ float relax_fwd(float P, int p, float s, float k, float b, float& bias) {
    const float pos = fmaxf(P, 0.f), neg = fminf(P, 0.f);
    if (p == 0) {
        bias += neg * b;
        return pos * s + neg * k;
    }
    bias += pos * b;
    return pos * k + neg * s;
}

// Same with a lower intercept bl (Sigmoid): lower bias P+ bl + P- b, upper
// bias P+ b + P- bl (BoundedSigmoidNode.cpp:723-799).
__device__ __forceinline__ float relax_fwd_bl(float P, int p, float s, float k, float b, float bl, float& bias) {
    const float pos = fmaxf(P, 0.f), neg = fminf(P, 0.f);
    if (p == 0) {
        bias += pos * bl + neg * b;
        return pos * s + neg * k;
    }
    bias += pos * b + neg * bl;
    return pos * k + neg * s;
}

__device__ __forceinline__ float relax_any(const ReluParams& rp, size_t bj, float P, int p, float s, float& bias) {
    if (rp.b_lo) return relax_fwd_bl(P, p, s, rp.k_up[bj], rp.b_up[bj], rp.b_lo[bj], bias);
    return relax_fwd(P, p, s, rp.k_up[bj], rp.b_up[bj], bias);
}

__device__ __forceinline__ float lower_slope(const ReluParams& rp, const float* alpha, int r, int bx,
                                             int j, int ncols) {
    const size_t bj = (size_t)bx * rp.n + j;
    if (alpha && (rp.flags[bj] & RF_USE_ALPHA)) return alpha[(size_t)r * ncols + j];
    return rp.slope_lo[bj];
}

// ============================================================== start step
__global__ void start_step_kernel(StartStep st) {
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= st.M) return;
    const int r = (int)warp;
    int p, rr;
    split_row(r, st.rows.R, p, rr);
    const int bx = st.rows.row_box[rr];
    const int id = st.rows.row_id[rr];
    const float* crow = nullptr;
    if (st.C) crow = st.C + ((size_t)(st.c_per_box ? bx : 0) * st.nspec + id) * st.spec_dim;
    float bias0 = 0.f;
    if (lane == 0) {
        if (crow) {
            for (int k = 0; k < st.spec_dim; ++k) bias0 = fmaf(crow[k], st.bW[k], bias0);
        } else {
            bias0 = st.bW[id];
        }
    }
    float part = 0.f;
    for (int c = lane; c < st.n; c += 32) {
        float P;
        if (crow) {
            P = 0.f;
            for (int k = 0; k < st.spec_dim; ++k) P = fmaf(crow[k], st.W[(size_t)k * st.n + c], P);
        } else {
            P = st.W[(size_t)id * st.n + c];
        }
        if (st.P_save) st.P_save[(size_t)r * st.n + c] = P;
        float Q = P;
        if (st.rp.n > 0) {
            const size_t bj = (size_t)bx * st.rp.n + c;
            const float s = lower_slope(st.rp, st.alpha, r, bx, c, st.n);
            Q = relax_any(st.rp, bj, P, p, s, part);
        }
        if (st.Q) st.Q[(size_t)r * st.n + c] = Q;
        if (st.b_next) part = fmaf(Q, st.b_next[c], part);
    }
    part = warp_sum(part);
    if (lane == 0) st.bias_acc[r] = bias0 + part;
}

void launch_start_step(const StartStep& st, cudaStream_t s) {
    if (st.M == 0) return;
    start_step_kernel<<<ceil_div((int64_t)st.M * 32, 256), 256, 0, s>>>(st);
    LB_LAUNCH();
}

// ============================================================== GEMM
// C = A . B, A [M,K] row-major, B [K,N] row-major, fp32 FMA.  128x128 tile
// per 256-thread CTA, 8x8 outputs per thread, K step 8.
constexpr int GBM = 128, GBN = 128, GBK = 8;

int gemm_tiles_n(int N) { return ceil_div(N, GBN); }

struct EpiFwdOp {
    EpiRelaxFwd e;
    int M, N;
    __device__ void operator()(int r0, int c0, float (&acc)[8][8], float (&part)[8]) const {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            part[i] = 0.f;
            if (r >= M) continue;
            int p, rr;
            split_row(r, e.rows.R, p, rr);
            const int bx = e.rows.row_box[rr];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j;
                if (c >= N) continue;
                const float P = acc[i][j];
                if (e.P_save) e.P_save[(size_t)r * N + c] = P;
                const size_t bj = (size_t)bx * e.rp.n + c;
                const float s = lower_slope(e.rp, e.alpha, r, bx, c, N);
                const float Q = relax_any(e.rp, bj, P, p, s, part[i]);
                e.Q[(size_t)r * N + c] = Q;
                if (e.b_next) part[i] = fmaf(Q, e.b_next[c], part[i]);
            }
        }
    }
};

struct EpiConcOp {
    EpiConcretize e;
    int M, N;
    __device__ void operator()(int r0, int c0, float (&acc)[8][8], float (&part)[8]) const {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            part[i] = 0.f;
            if (r >= M) continue;
            int p, rr;
            split_row(r, e.rows.R, p, rr);
            const int bx = e.rows.row_box[rr];
            const float* xa = (p == 0 ? e.xl : e.xu) + (size_t)bx * N;
            const float* xb = (p == 0 ? e.xu : e.xl) + (size_t)bx * N;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j;
                if (c >= N) continue;
                const float P = acc[i][j];
                part[i] += fmaxf(P, 0.f) * xa[c] + fminf(P, 0.f) * xb[c];
                if (e.sign)
                    e.sign[(size_t)r * N + c] = (uint8_t)((P >= 0.f ? 1 : 0) | (P <= 0.f ? 2 : 0));
            }
        }
    }
};

template <bool SIG>
struct EpiAdjOp {
    EpiRelaxAdj e;
    int M, N;
    // Flush the running sums of one (8-row group, virtual box) segment.
    __device__ void flush(int rg, int vb, int c0, const float (&kacc)[8], const float (&bacc)[8],
                          const float (&sacc)[8], const float (&blacc)[8]) const {
        const size_t slot = (size_t)(rg + vb) * N;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = c0 + j;
            if (c < N) {
                e.kslot[slot + c] = kacc[j];
                e.bslot[slot + c] = bacc[j];
                if (SIG) {
                    e.sslot[slot + c] = sacc[j];
                    e.blslot[slot + c] = blacc[j];
                }
            }
        }
    }
    __device__ void operator()(int r0, int c0, float (&acc)[8][8], float (&part)[8]) const {
        float kacc[8], bacc[8], sacc[8], blacc[8];
        int cur_vb = -1;
        const int rg = r0 >> 3;
#pragma unroll
        for (int j = 0; j < 8; ++j) kacc[j] = bacc[j] = sacc[j] = blacc[j] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            part[i] = 0.f;
            if (r >= M) continue;
            int p, rr;
            split_row(r, e.rows.R, p, rr);
            const int bx = e.rows.row_box[rr];
            const int vb = bx + p * e.B;
            if (vb != cur_vb) {
                if (cur_vb >= 0) {
                    flush(rg, cur_vb, c0, kacc, bacc, sacc, blacc);
#pragma unroll
                    for (int j = 0; j < 8; ++j) kacc[j] = bacc[j] = sacc[j] = blacc[j] = 0.f;
                }
                cur_vb = vb;
            }
            const float g = e.gseed[r];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j;
                if (c >= N) continue;
                const float Qbar = acc[i][j] + g * e.b_lin[c];
                // P of the ReLU below a one-hot start is its weight row when
                // the forward pass gathered it instead of saving it.
                const float P = e.gather_W ? e.gather_W[(size_t)e.rows.row_id[rr] * N + c]
                                           : e.P_saved[(size_t)r * N + c];
                const size_t bj = (size_t)bx * e.rp.n + c;
                const uint8_t f = e.rp.flags[bj];
                const float s = lower_slope(e.rp, e.alpha, r, bx, c, N);
                const float k = e.rp.k_up[bj], b = e.rp.b_up[bj];
                const float bl = SIG ? e.rp.b_lo[bj] : 0.f;
                const bool pos = P >= 0.f, neg = P <= 0.f;
                const float sP = p == 0 ? s : k, sN = p == 0 ? k : s;
                const float bP = p == 0 ? bl : b, bN = p == 0 ? b : bl;
                if (e.Pbar) {
                    const float dq = (pos ? sP : 0.f) + (neg ? sN : 0.f);
                    const float db = (pos ? bP : 0.f) + (neg ? bN : 0.f);
                    e.Pbar[(size_t)r * N + c] = Qbar * dq + g * db;
                }
                const float Pp = fmaxf(P, 0.f), Pn = fminf(P, 0.f);
                const float ag = (f & RF_USE_ALPHA) ? Qbar * (p == 0 ? Pp : Pn) : 0.f;
                if (e.adam_m) {
                    if (e.active[bx]) {
                        const size_t at = (size_t)r * N + c;
                        float mm = e.adam_m[at], vv = e.adam_v[at];
                        e.alpha[at] = adam_clip_update(e.alpha[at], ag, mm, vv, e.adam_step, e.adam_bc2_sqrt);
                        e.adam_m[at] = mm;
                        e.adam_v[at] = vv;
                    }
                } else if (e.alpha_grad) {
                    e.alpha_grad[(size_t)r * N + c] = ag;
                }
                if (f & RF_UNSTABLE) {
                    kacc[j] += Qbar * (p == 0 ? Pn : Pp);
                    bacc[j] += g * (p == 0 ? Pn : Pp);
                    if (SIG) {
                        sacc[j] += Qbar * (p == 0 ? Pp : Pn);
                        blacc[j] += g * (p == 0 ? Pp : Pn);
                    }
                }
            }
        }
        if (cur_vb >= 0) flush(rg, cur_vb, c0, kacc, bacc, sacc, blacc);
    }
};

template <class Epi>
__global__ void __launch_bounds__(256) gemm_kernel(const float* __restrict__ A,
                                                   const float* __restrict__ Bm, int M, int N, int K,
                                                   bool vecA, bool vecB, Epi epi,
                                                   float* __restrict__ partial) {
    __shared__ __align__(16) float As[GBK][GBM + 4];
    __shared__ __align__(16) float Bs[GBK][GBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    const int a_row = tid >> 1, a_k = (tid & 1) * 4;
    const int b_k = tid >> 5, b_col = (tid & 31) * 4;
    for (int k0 = 0; k0 < K; k0 += GBK) {
        {
            const int gr = m0 + a_row, gk = k0 + a_k;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (gr < M) {
                const float* src = A + (size_t)gr * K + gk;
                if (vecA && gk + 3 < K) {
                    const float4 t = *reinterpret_cast<const float4*>(src);
                    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (gk + q < K) v[q] = src[q];
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) As[a_k + q][a_row] = v[q];
        }
        {
            const int gk = k0 + b_k, gc = n0 + b_col;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (gk < K) {
                const float* src = Bm + (size_t)gk * N + gc;
                if (vecB && gc + 3 < N) {
                    const float4 t = *reinterpret_cast<const float4*>(src);
                    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (gc + q < N) v[q] = src[q];
                }
            }
            *reinterpret_cast<float4*>(&Bs[b_k][b_col]) = make_float4(v[0], v[1], v[2], v[3]);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < GBK; ++kk) {
            float a[8], b[8];
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8 + 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
    float part[8];
    epi(m0 + ty * 8, n0 + tx * 8, acc, part);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float v = part[i];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, 16);
        const int r = m0 + ty * 8 + i;
        if (tx == 0 && r < M && partial) partial[(size_t)blockIdx.x * M + r] = v;
    }
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <class Op>
static void run_gemm(const float* A, const float* Bm, int M, int N, int K, const Op& op,
                     float* partial, cudaStream_t s) {
    if (M == 0 || N == 0) return;
    dim3 grid(ceil_div(N, GBN), ceil_div(M, GBM));
    const bool vecA = (K % 4 == 0) && aligned16(A);
    const bool vecB = (N % 4 == 0) && aligned16(Bm);
    gemm_kernel<Op><<<grid, 256, 0, s>>>(A, Bm, M, N, K, vecA, vecB, op, partial);
    LB_LAUNCH();
}

void launch_gemm_relax_fwd(const float* A, const float* Bm, int M, int N, int K,
                           const EpiRelaxFwd& e, float* partial, cudaStream_t s) {
    run_gemm(A, Bm, M, N, K, EpiFwdOp{e, M, N}, partial, s);
}
void launch_gemm_concretize(const float* A, const float* Bm, int M, int N, int K,
                            const EpiConcretize& e, float* partial, cudaStream_t s) {
    run_gemm(A, Bm, M, N, K, EpiConcOp{e, M, N}, partial, s);
}
void launch_gemm_relax_adj(const float* A, const float* Bm, int M, int N, int K,
                           const EpiRelaxAdj& e, float* partial, cudaStream_t s) {
    if (e.rp.b_lo)
        run_gemm(A, Bm, M, N, K, EpiAdjOp<true>{e, M, N}, partial, s);
    else
        run_gemm(A, Bm, M, N, K, EpiAdjOp<false>{e, M, N}, partial, s);
}

// One CTA per (box, 32-column chunk); 256 threads = 32 columns x 8 row lanes.
// Walks the box's rows of both sides; column sums of the k_up / b_up
// adjoints go through shared memory in a fixed order.
__global__ void __launch_bounds__(256) relax_adjoint_kernel(EpiRelaxAdj e, const float* __restrict__ Qbar,
                                                            int M, int n) {
    const int bx = blockIdx.x;
    const int c = blockIdx.y * 32 + (threadIdx.x & 31);
    const int ty = threadIdx.x >> 5;
    __shared__ float sk[8][32], sb[8][32];
    float ks = 0.f, bs = 0.f;
    if (c < n) {
        const size_t bj = (size_t)bx * e.rp.n + c;
        const uint8_t f = e.rp.flags[bj];
        const float sl = e.rp.slope_lo[bj], k = e.rp.k_up[bj], b = e.rp.b_up[bj];
        const bool use_alpha = (f & RF_USE_ALPHA) != 0, un = (f & RF_UNSTABLE) != 0;
        const bool act = e.active ? e.active[bx] != 0 : false;
        for (int p = 0; p < 2; ++p) {
            const int first = p * e.rows.R + e.rows.box_off[bx];
            const int last = min(p * e.rows.R + e.rows.box_off[bx + 1], M);
            for (int r = first + ty; r < last; r += 8) {
                const size_t at = (size_t)r * n + c;
                const float Qb = Qbar[at];
                const float P = e.gather_W ? e.gather_W[(size_t)e.rows.row_id[r - p * e.rows.R] * n + c]
                                           : e.P_saved[at];
                const float g = e.gseed[r];
                const bool adam = e.adam_m && act && (f & RF_ASET);
                const float a = (e.alpha && (use_alpha || adam)) ? e.alpha[at] : 0.f;
                const float s = (e.alpha && use_alpha) ? a : sl;
                const bool pos = P >= 0.f, neg = P <= 0.f;
                const float sP = p == 0 ? s : k, sN = p == 0 ? k : s;
                const float bP = p == 0 ? 0.f : b, bN = p == 0 ? b : 0.f;
                if (e.Pbar) {
                    const float dq = (pos ? sP : 0.f) + (neg ? sN : 0.f);
                    const float db = (pos ? bP : 0.f) + (neg ? bN : 0.f);
                    e.Pbar[e.ps.s ? phase_dst(e.ps, r, c) : (int64_t)at] = Qb * dq + g * db;
                }
                const float Pp = fmaxf(P, 0.f), Pn = fminf(P, 0.f);
                if (un) {
                    ks += Qb * (p == 0 ? Pn : Pp);
                    bs += g * (p == 0 ? Pn : Pp);
                }
                if (adam) {
                    const float ag = use_alpha ? Qb * (p == 0 ? Pp : Pn) : 0.f;
                    float mm = e.adam_m[at], vv = e.adam_v[at];
                    e.alpha[at] = adam_clip_update(a, ag, mm, vv, e.adam_step, e.adam_bc2_sqrt);
                    e.adam_m[at] = mm;
                    e.adam_v[at] = vv;
                }
            }
        }
    }
    sk[ty][threadIdx.x & 31] = ks;
    sb[ty][threadIdx.x & 31] = bs;
    __syncthreads();
    if (ty == 0 && c < n) {
        float kt = 0.f, bt = 0.f;
        for (int q = 0; q < 8; ++q) {
            kt += sk[q][threadIdx.x];
            bt += sb[q][threadIdx.x];
        }
        e.kbar[(size_t)bx * n + c] += kt;
        e.bbar[(size_t)bx * n + c] += bt;
    }
}

// Vectorised variant (n % 4 == 0): one CTA per (box, 128 columns); 256
// threads = 32 column lanes of 4 columns x 8 row lanes; float4 traffic.
// CT column threads x (256 / CT) row lanes per block, 4 columns per thread.
template <int CT>
__global__ void __launch_bounds__(256, 3) relax_adjoint_v4_kernel(EpiRelaxAdj e, const float* __restrict__ Qbar,
                                                               int M, int n) {
    constexpr int RL = 256 / CT;
    const int bx = blockIdx.x;
    const int c = blockIdx.y * (4 * CT) + (threadIdx.x % CT) * 4;
    const int ty = threadIdx.x / CT;
    __shared__ float4 sk[RL][CT], sb[RL][CT];
    float ks[4] = {0.f, 0.f, 0.f, 0.f}, bs[4] = {0.f, 0.f, 0.f, 0.f};
    const float* __restrict__ Ps = e.P_saved;
    const float* __restrict__ Gw = e.gather_W;
    const float* __restrict__ gs = e.gseed;
    float* __restrict__ al = e.alpha;
    float* __restrict__ am = e.adam_m;
    float* __restrict__ av = e.adam_v;
    float* __restrict__ pb = e.Pbar;
    if (c < n) {
        const size_t bj = (size_t)bx * e.rp.n + c;
        float sl[4], ku[4], bu[4];
        const float4 sl4 = *reinterpret_cast<const float4*>(e.rp.slope_lo + bj);
        const float4 ku4 = *reinterpret_cast<const float4*>(e.rp.k_up + bj);
        const float4 bu4 = *reinterpret_cast<const float4*>(e.rp.b_up + bj);
        const uchar4 f4 = *reinterpret_cast<const uchar4*>(e.rp.flags + bj);
        sl[0] = sl4.x; sl[1] = sl4.y; sl[2] = sl4.z; sl[3] = sl4.w;
        ku[0] = ku4.x; ku[1] = ku4.y; ku[2] = ku4.z; ku[3] = ku4.w;
        bu[0] = bu4.x; bu[1] = bu4.y; bu[2] = bu4.z; bu[3] = bu4.w;
        const uint8_t fl[4] = {f4.x, f4.y, f4.z, f4.w};
        const bool act = e.active ? e.active[bx] != 0 : false;
        // Alphas outside the creation set never move (zero gradient, zero
        // moments): their 4-column group skips the Adam traffic.
        const bool adam = am != nullptr && act && ((fl[0] | fl[1] | fl[2] | fl[3]) & RF_ASET);
        const bool need_alpha = al != nullptr && (adam || ((fl[0] | fl[1] | fl[2] | fl[3]) & RF_USE_ALPHA));
        // Column part of the Pbar address (fixed for this thread).
        const int64_t pcol = (pb && e.ps.s) ? phase_dst(e.ps, 0, c) : (int64_t)c;
        const int64_t pstride = e.ps.s ? e.ps.row_stride : (int64_t)n;
        for (int p = 0; p < 2; ++p) {
            const int first = p * e.rows.R + e.rows.box_off[bx];
            const int last = min(p * e.rows.R + e.rows.box_off[bx + 1], M);
#pragma unroll 2
            for (int r = first + ty; r < last; r += RL) {
                const size_t at = (size_t)r * n + c;
                const float4 q4 = *reinterpret_cast<const float4*>(Qbar + at);
                const float4 p4 = Gw ? *reinterpret_cast<const float4*>(Gw + (size_t)e.rows.row_id[r - p * e.rows.R] * n + c)
                                     : *reinterpret_cast<const float4*>(Ps + at);
                const float g = gs[r];
                float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (need_alpha) a4 = *reinterpret_cast<const float4*>(al + at);
                float4 m4, v4;
                if (adam) {
                    m4 = *reinterpret_cast<const float4*>(am + at);
                    v4 = *reinterpret_cast<const float4*>(av + at);
                }
                const float Q[4] = {q4.x, q4.y, q4.z, q4.w};
                const float P[4] = {p4.x, p4.y, p4.z, p4.w};
                float A[4] = {a4.x, a4.y, a4.z, a4.w};
                float Mm[4] = {0.f, 0.f, 0.f, 0.f}, Vv[4] = {0.f, 0.f, 0.f, 0.f};
                if (adam) {
                    Mm[0] = m4.x; Mm[1] = m4.y; Mm[2] = m4.z; Mm[3] = m4.w;
                    Vv[0] = v4.x; Vv[1] = v4.y; Vv[2] = v4.z; Vv[3] = v4.w;
                }
                float out[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const bool use_alpha = (fl[i] & RF_USE_ALPHA) != 0, un = (fl[i] & RF_UNSTABLE) != 0;
                    const float s = (al && use_alpha) ? A[i] : sl[i];
                    const bool pos = P[i] >= 0.f, neg = P[i] <= 0.f;
                    const float sP = p == 0 ? s : ku[i], sN = p == 0 ? ku[i] : s;
                    const float bP = p == 0 ? 0.f : bu[i], bN = p == 0 ? bu[i] : 0.f;
                    const float dq = (pos ? sP : 0.f) + (neg ? sN : 0.f);
                    const float db = (pos ? bP : 0.f) + (neg ? bN : 0.f);
                    out[i] = Q[i] * dq + g * db;
                    const float Pp = fmaxf(P[i], 0.f), Pn = fminf(P[i], 0.f);
                    if (un) {
                        ks[i] += Q[i] * (p == 0 ? Pn : Pp);
                        bs[i] += g * (p == 0 ? Pn : Pp);
                    }
                    if (adam) {
                        const float ag = use_alpha ? Q[i] * (p == 0 ? Pp : Pn) : 0.f;
                        A[i] = adam_clip_update(A[i], ag, Mm[i], Vv[i], e.adam_step, e.adam_bc2_sqrt);
                    }
                }
                if (pb)
                    *reinterpret_cast<float4*>(pb + (int64_t)r * pstride + pcol) =
                        make_float4(out[0], out[1], out[2], out[3]);
                if (adam) {
                    *reinterpret_cast<float4*>(al + at) = make_float4(A[0], A[1], A[2], A[3]);
                    *reinterpret_cast<float4*>(am + at) = make_float4(Mm[0], Mm[1], Mm[2], Mm[3]);
                    *reinterpret_cast<float4*>(av + at) = make_float4(Vv[0], Vv[1], Vv[2], Vv[3]);
                }
            }
        }
    }
    sk[ty][threadIdx.x % CT] = make_float4(ks[0], ks[1], ks[2], ks[3]);
    sb[ty][threadIdx.x % CT] = make_float4(bs[0], bs[1], bs[2], bs[3]);
    __syncthreads();
    if (ty == 0 && c < n) {
        float4 kt = make_float4(0.f, 0.f, 0.f, 0.f), bt = kt;
        for (int q = 0; q < RL; ++q) {
            const float4 a = sk[q][threadIdx.x], b = sb[q][threadIdx.x];
            kt.x += a.x; kt.y += a.y; kt.z += a.z; kt.w += a.w;
            bt.x += b.x; bt.y += b.y; bt.z += b.z; bt.w += b.w;
        }
        float4* kp = reinterpret_cast<float4*>(e.kbar + (size_t)bx * n + c);
        float4* bp = reinterpret_cast<float4*>(e.bbar + (size_t)bx * n + c);
        float4 k0 = *kp, b0 = *bp;
        k0.x += kt.x; k0.y += kt.y; k0.z += kt.z; k0.w += kt.w;
        b0.x += bt.x; b0.y += bt.y; b0.z += bt.z; b0.w += bt.w;
        *kp = k0;
        *bp = b0;
    }
}

void launch_relax_adjoint(const EpiRelaxAdj& e, const float* Qbar, int M, int n, cudaStream_t s) {
    if (M == 0 || e.B == 0) return;
    if (n % 4 == 0) {
        // 64 columns per block: twice the blocks of 128-column ones, so the
        // boxes' uneven row counts leave a shorter tail.
        dim3 grid(e.B, ceil_div(n, 64));
        relax_adjoint_v4_kernel<16><<<grid, 256, 0, s>>>(e, Qbar, M, n);
    } else {
        dim3 grid(e.B, ceil_div(n, 32));
        relax_adjoint_kernel<<<grid, 256, 0, s>>>(e, Qbar, M, n);
    }
    LB_LAUNCH();
}

int relax_grad_slots(int M, int B, int group) { return ceil_div(M, group) + 2 * B; }

// One thread per (box, column): the slots of virtual box vb cover the
// `group`-row groups from first_row/group to last_row/group, each at slot
// index (row group + vb).
__global__ void reduce_relax_grad_kernel(RowMap rows, int M, int B, int N, int group,
                                         const float* __restrict__ kslot, const float* __restrict__ bslot,
                                         float* __restrict__ kbar, float* __restrict__ bbar) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)B * N) return;
    const int bx = (int)(idx / N), c = (int)(idx % N);
    float ks = 0.f, bs = 0.f;
    for (int p = 0; p < 2; ++p) {
        const int first = p * rows.R + rows.box_off[bx];
        const int last = min(p * rows.R + rows.box_off[bx + 1], M);  // exclusive
        if (first >= last) continue;
        const int vb = bx + p * B;
        for (int g = first / group; g <= (last - 1) / group; ++g) {
            const size_t at = (size_t)(g + vb) * N + c;
            ks += kslot[at];
            bs += bslot[at];
        }
    }
    kbar[idx] += ks;
    bbar[idx] += bs;
}

void launch_reduce_relax_grad(const RowMap& rows, int M, int B, int N, int group, const float* kslot,
                              const float* bslot, float* kbar, float* bbar, cudaStream_t s) {
    if ((int64_t)B * N == 0 || M == 0) return;
    reduce_relax_grad_kernel<<<ceil_div((int64_t)B * N, 256), 256, 0, s>>>(rows, M, B, N, group, kslot, bslot,
                                                                           kbar, bbar);
    LB_LAUNCH();
}

__global__ void sum_partials_kernel(const float* __restrict__ base, const float* __restrict__ partial,
                                    int ntiles, int M, float* __restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= M) return;
    float v = base ? base[r] : 0.f;
    for (int t = 0; t < ntiles; ++t) v += partial[(size_t)t * M + r];
    out[r] = v;
}

void launch_sum_partials(const float* base, const float* partial, int ntiles, int M, float* out,
                         cudaStream_t s) {
    if (M == 0) return;
    sum_partials_kernel<<<ceil_div(M, 256), 256, 0, s>>>(base, partial, ntiles, M, out);
    LB_LAUNCH();
}

// ============================================================== finalisation
__global__ void scatter_start_kernel(RowMap rows, const float* __restrict__ val,
                                     const float* __restrict__ ref_l, const float* __restrict__ ref_u,
                                     int n, float* __restrict__ cur_l, float* __restrict__ cur_u) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    const size_t at = (size_t)rows.row_box[r] * n + rows.row_id[r];
    float lo = val[r], hi = val[rows.R + r];
    if (ref_l) {
        // CROWNAnalysis::concretizeNode STE clamp (:921-938), value part.
        lo = (fmaxf(ref_l[at], lo) - lo) + lo;
        hi = hi - (hi - fminf(ref_u[at], hi));
    }
    cur_l[at] = lo;
    cur_u[at] = hi;
}

void launch_scatter_start(const RowMap& rows, const float* val, const float* ref_l,
                          const float* ref_u, int n, float* cur_l, float* cur_u, cudaStream_t s) {
    if (rows.R == 0) return;
    scatter_start_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, val, ref_l, ref_u, n, cur_l, cur_u);
    LB_LAUNCH();
}

__global__ void scatter_output_kernel(RowMap rows, const float* __restrict__ val, int nspec,
                                      bool has_upper, float* __restrict__ lb, float* __restrict__ ub) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    const size_t at = (size_t)rows.row_box[r] * nspec + rows.row_id[r];
    lb[at] = val[r];
    if (has_upper) ub[at] = val[rows.R + r];
}

void launch_scatter_output(const RowMap& rows, const float* val, int nspec, bool has_upper,
                           float* lb, float* ub, cudaStream_t s) {
    if (rows.R == 0) return;
    scatter_output_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, val, nspec, has_upper, lb, ub);
    LB_LAUNCH();
}

// ============================================================== control
__global__ void alpha_control_kernel(BoxControl c, const float* __restrict__ cur, const float* __restrict__ verify,
                                     int B, int nspec, int iter, int save_after, int patience_limit, bool has_loss) {
    const int bx = blockIdx.x * blockDim.x + threadIdx.x;
    if (bx >= B) return;
    c.save[bx] = 0;
    if (!c.active[bx]) return;
    const float* cv = cur + (size_t)bx * nspec;
    float* best = c.best + (size_t)bx * nspec;
    uint8_t* imp = c.improved + (size_t)bx * nspec;
    const float* vv = verify ? verify + (size_t)bx * nspec : cv;
    if (c.thr && lb200::box_verified(vv, c.thr, c.branch, nspec, c.n_branches)) {
        // Verified during the optimisation (AlphaCROWNAnalysis.cpp:396-407):
        // the best bound takes this iteration's, nothing is saved, the box
        // stops.
        for (int j = 0; j < nspec; ++j) best[j] = c.has_best[bx] ? fmaxf(best[j], cv[j]) : cv[j];
        c.has_best[bx] = 1;
        c.active[bx] = 0;
        return;
    }
    bool any = false;
    if (!c.has_best[bx]) {
        for (int j = 0; j < nspec; ++j) {
            best[j] = cv[j];
            imp[j] = 1;
        }
        c.has_best[bx] = 1;
        any = nspec > 0;
    } else {
        for (int j = 0; j < nspec; ++j) {
            const bool b = cv[j] > best[j];
            imp[j] = b ? 1 : 0;
            any |= b;
        }
        if (any)
            for (int j = 0; j < nspec; ++j) best[j] = fmaxf(best[j], cv[j]);
    }
    const int pat = c.patience[bx];
    const bool save = any && (iter < 1 || iter > save_after || pat >= patience_limit);
    c.save[bx] = save ? 1 : 0;
    float loss = 0.f;
    if (has_loss) {
        for (int j = 0; j < nspec; ++j) loss += cv[j];
        loss = fabsf(-loss);
    }
    if (any) {
        if (has_loss) c.best_loss[bx] = loss;
        c.patience[bx] = 0;
    } else if (has_loss) {
        if (loss < c.best_loss[bx]) {
            c.best_loss[bx] = loss;
            c.patience[bx] = 0;
        } else {
            c.patience[bx] = pat + 1;
        }
    }
    if (c.patience[bx] >= patience_limit) c.active[bx] = 0;
    else if (c.n_active) atomicAdd(c.n_active, 1);
}

__global__ void crown_verified_kernel(const float* __restrict__ lb, const float* __restrict__ thr,
                                      const int32_t* __restrict__ branch, int n_branches, int B, int nspec,
                                      int* __restrict__ done, int* __restrict__ active, int* n_done) {
    const int bx = blockIdx.x * blockDim.x + threadIdx.x;
    if (bx >= B) return;
    const bool v = lb200::box_verified(lb + (size_t)bx * nspec, thr, branch, nspec, n_branches);
    done[bx] = v ? 1 : 0;
    active[bx] = v ? 0 : 1;
    if (v) atomicAdd(n_done, 1);
}

void launch_crown_verified(const float* lb, const float* thr, const int32_t* branch, int n_branches, int B,
                           int nspec, int* done, int* active, int* n_done, cudaStream_t s) {
    crown_verified_kernel<<<ceil_div(B, 128), 128, 0, s>>>(lb, thr, branch, n_branches, B, nspec, done, active,
                                                           n_done);
    LB_LAUNCH();
}

__global__ void take_verified_kernel(const int* __restrict__ done, const float* __restrict__ crown_lb,
                                     const float* __restrict__ crown_ub, int B, int nspec, float* __restrict__ lb,
                                     float* __restrict__ ub) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)B * nspec) return;
    if (!done[idx / nspec]) return;
    lb[idx] = crown_lb[idx];
    ub[idx] = crown_ub[idx];
}

void launch_take_verified(const int* done, const float* crown_lb, const float* crown_ub, int B, int nspec,
                          float* lb, float* ub, cudaStream_t s) {
    take_verified_kernel<<<ceil_div((int64_t)B * nspec, 256), 256, 0, s>>>(done, crown_lb, crown_ub, B, nspec, lb,
                                                                           ub);
    LB_LAUNCH();
}

void launch_alpha_control(const BoxControl& c, const float* cur, const float* verify, int B, int nspec, int iter,
                          int save_after, int patience_limit, bool has_loss, cudaStream_t s) {
    alpha_control_kernel<<<ceil_div(B, 128), 128, 0, s>>>(c, cur, verify, B, nspec, iter, save_after,
                                                          patience_limit, has_loss);
    LB_LAUNCH();
}

__global__ void snapshot_kernel(const int* __restrict__ save, const float* __restrict__ cur_l,
                                const float* __restrict__ cur_u, int B, int n,
                                float* __restrict__ best_l, float* __restrict__ best_u) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)B * n) return;
    if (!save[idx / n]) return;
    best_l[idx] = fmaxf(best_l[idx], cur_l[idx]);
    best_u[idx] = fminf(best_u[idx], cur_u[idx]);
}

void launch_snapshot(const int* save, const float* cur_l, const float* cur_u, int B, int n,
                     float* best_l, float* best_u, cudaStream_t s) {
    snapshot_kernel<<<ceil_div((int64_t)B * n, 256), 256, 0, s>>>(save, cur_l, cur_u, B, n, best_l, best_u);
    LB_LAUNCH();
}

__global__ void best_alpha_kernel(RowMap rows, const int* __restrict__ save,
                                  const int* __restrict__ first_save, const uint8_t* __restrict__ improved,
                                  int nspec, int n, const float* __restrict__ alpha,
                                  float* __restrict__ best) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)2 * rows.R * n) return;
    const int r2 = (int)(idx / n);
    const int rr = r2 >= rows.R ? r2 - rows.R : r2;
    const int bx = rows.row_box[rr];
    if (!save[bx]) return;
    bool copy = first_save[bx] != 0;
    if (!copy) {
        const int local = rr - rows.box_off[bx];
        copy = local < nspec && improved[(size_t)bx * nspec + local];
    }
    if (copy) best[idx] = alpha[idx];
}

void launch_best_alpha(const RowMap& rows, const int* save, const int* first_save,
                       const uint8_t* improved, int nspec, int n, const float* alpha,
                       float* best_alpha, cudaStream_t s) {
    const int64_t total = (int64_t)2 * rows.R * n;
    if (total == 0) return;
    best_alpha_kernel<<<ceil_div(total, 256), 256, 0, s>>>(rows, save, first_save, improved, nspec,
                                                           n, alpha, best_alpha);
    LB_LAUNCH();
}

// Block row y = (side, box, local row < nspec); x = 1024 columns.
__global__ void best_alpha_rows_kernel(RowMap rows, int B, const int* __restrict__ save,
                                       const uint8_t* __restrict__ improved, int nspec, int n,
                                       const float* __restrict__ alpha, float* __restrict__ best) {
    for (int y = blockIdx.y; y < 2 * B * nspec; y += gridDim.y) {
        const int p = y / (B * nspec), rem = y - p * (B * nspec);
        const int bx = rem / nspec, local = rem - bx * nspec;
        if (!save[bx] || !improved[(size_t)bx * nspec + local]) continue;
        const int first = rows.box_off[bx];
        if (first + local >= rows.box_off[bx + 1]) continue;
        const size_t row = (size_t)p * rows.R + first + local;
        copy_row(alpha + row * n, best + row * n, n);
    }
}

void launch_best_alpha_rows(const RowMap& rows, int B, const int* save, const uint8_t* improved, int nspec,
                            int n, const float* alpha, float* best_alpha, cudaStream_t s) {
    if (B == 0 || nspec == 0 || n == 0 || rows.R == 0) return;
    const dim3 grid(ceil_div(n, 1024), std::min(2 * B * nspec, 65535));
    best_alpha_rows_kernel<<<grid, 256, 0, s>>>(rows, B, save, improved, nspec, n, alpha, best_alpha);
    LB_LAUNCH();
}

__global__ void clear_first_save_kernel(const int* save, int* first_save, int B) {
    const int bx = blockIdx.x * blockDim.x + threadIdx.x;
    if (bx < B && save[bx]) first_save[bx] = 0;
}

void launch_clear_first_save(const int* save, int* first_save, int B, cudaStream_t s) {
    clear_first_save_kernel<<<ceil_div(B, 256), 256, 0, s>>>(save, first_save, B);
    LB_LAUNCH();
}

// torch::optim::Adam step (exp_avg = exp_avg*b1 + (1-b1) g; exp_avg_sq =
// exp_avg_sq*b2 + (1-b2) g g; p += -step * exp_avg / (sqrt(exp_avg_sq)/sqrt(bc2) + eps))
// followed by the [0, 1] clamp of AlphaCROWNAnalysis::clipAlphaParameters.
__global__ void adam_kernel(RowMap rows, const int* __restrict__ active, int n,
                            float* __restrict__ alpha, float* __restrict__ m, float* __restrict__ v,
                            const float* __restrict__ grad, float step_size, float bc2_sqrt) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)2 * rows.R * n) return;
    const int r2 = (int)(idx / n);
    const int rr = r2 >= rows.R ? r2 - rows.R : r2;
    if (!active[rows.row_box[rr]]) return;
    float mm = m[idx], vv = v[idx];
    alpha[idx] = adam_clip_update(alpha[idx], grad[idx], mm, vv, step_size, bc2_sqrt);
    m[idx] = mm;
    v[idx] = vv;
}

void launch_adam(const RowMap& rows, const int* active, int n, float* alpha, float* m, float* v,
                 const float* grad, float step_size, float bc2_sqrt, cudaStream_t s) {
    const int64_t total = (int64_t)2 * rows.R * n;
    if (total == 0) return;
    adam_kernel<<<ceil_div(total, 256), 256, 0, s>>>(rows, active, n, alpha, m, v, grad, step_size,
                                                     bc2_sqrt);
    LB_LAUNCH();
}

__global__ void max_best_kernel(const float* __restrict__ best, const int* __restrict__ has_best,
                                int total, int nspec, float* __restrict__ lb) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    if (has_best[i / nspec]) lb[i] = fmaxf(lb[i], best[i]);
}

void launch_max_best(const float* best, const int* has_best, int total, int nspec, float* lb,
                     cudaStream_t s) {
    if (total == 0) return;
    max_best_kernel<<<ceil_div(total, 256), 256, 0, s>>>(best, has_best, total, nspec, lb);
    LB_LAUNCH();
}

// ============================================================== adjoint
__global__ void adj_input_seed_kernel(RowMap rows, int M, const uint8_t* __restrict__ sign,
                                      const float* __restrict__ g, const float* __restrict__ xl,
                                      const float* __restrict__ xu, int n0, float* __restrict__ out) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)M * n0) return;
    const int r = (int)(idx / n0), j = (int)(idx % n0);
    int p, rr;
    split_row(r, rows.R, p, rr);
    const int bx = rows.row_box[rr];
    const float xa = (p == 0 ? xl : xu)[(size_t)bx * n0 + j];
    const float xb = (p == 0 ? xu : xl)[(size_t)bx * n0 + j];
    const uint8_t sg = sign[idx];
    const float gr = g[r];
    out[idx] = ((sg & 1) ? gr * xa : 0.f) + ((sg & 2) ? gr * xb : 0.f);
}

void launch_adj_input_seed(const RowMap& rows, int M, const uint8_t* sign, const float* g,
                           const float* xl, const float* xu, int n0, float* Pbar0, cudaStream_t s) {
    const int64_t total = (int64_t)M * n0;
    if (total == 0) return;
    adj_input_seed_kernel<<<ceil_div(total, 256), 256, 0, s>>>(rows, M, sign, g, xl, xu, n0, Pbar0);
    LB_LAUNCH();
}

// d loss / d (l, u) of one unstable neuron through k_up = d and b_up = -l d,
// d = ub_r / (ub_r - lb_r), lb_r = min(l, 0), ub_r = max(max(u, 0), lb_r + 1e-8),
// following autograd's rules for clamp_max / clamp_min / maximum / div.
__global__ void bound_grad_kernel(RowMap rows, const float* __restrict__ cur_l,
                                  const float* __restrict__ cur_u, const uint8_t* __restrict__ flags,
                                  const float* __restrict__ kbar, const float* __restrict__ bbar,
                                  int n, float* __restrict__ g) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    const size_t at = (size_t)rows.row_box[r] * n + rows.row_id[r];
    float gl = 0.f, gu = 0.f;
    if (flags[at] & RF_UNSTABLE) {
        const float l = cur_l[at], u = cur_u[at];
        const float lb_r = fminf(l, 0.f);
        const float ub_r0 = fmaxf(u, 0.f);
        const float t = lb_r + 1e-8f;
        const float ub_r = fmaxf(ub_r0, t);
        const float den = ub_r - lb_r;
        const float d = ub_r / den;
        const float kb = kbar[at], bb = bbar[at];
        const float dbar = kb + bb * (-l);
        gl = bb * (-d);
        float ubr_bar = dbar / den;
        const float den_bar = -dbar * ub_r / (den * den);
        ubr_bar += den_bar;
        float lbr_bar = -den_bar;
        float ub0_bar = 0.f, t_bar = 0.f;
        if (ub_r0 > t) ub0_bar = ubr_bar;
        else if (t > ub_r0) t_bar = ubr_bar;
        else { ub0_bar = 0.5f * ubr_bar; t_bar = 0.5f * ubr_bar; }
        lbr_bar += t_bar;
        gu = (u >= 0.f) ? ub0_bar : 0.f;
        gl += (l <= 0.f) ? lbr_bar : 0.f;
    }
    g[r] = gl;
    g[rows.R + r] = gu;
}

void launch_bound_grad(const RowMap& rows, const float* cur_l, const float* cur_u,
                       const uint8_t* flags, const float* kbar, const float* bbar, int n, float* g,
                       cudaStream_t s) {
    if (rows.R == 0) return;
    bound_grad_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, cur_l, cur_u, flags, kbar, bbar, n, g);
    LB_LAUNCH();
}

__global__ void output_seed_kernel(RowMap rows, const int* __restrict__ active, float* __restrict__ g) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    g[r] = active[rows.row_box[r]] ? -1.f : 0.f;
}

void launch_output_seed(const RowMap& rows, const int* active, float* g, cudaStream_t s) {
    if (rows.R == 0) return;
    output_seed_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, active, g);
    LB_LAUNCH();
}

__global__ void output_seed_upper_kernel(RowMap rows, const int* __restrict__ active, float* __restrict__ g) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    g[r] = 0.f;
    g[rows.R + r] = active[rows.row_box[r]] ? 1.f : 0.f;
}

void launch_output_seed_upper(const RowMap& rows, const int* active, float* g, cudaStream_t s) {
    if (rows.R == 0) return;
    output_seed_upper_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, active, g);
    LB_LAUNCH();
}

__global__ void negate_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = -in[i];
}

void launch_negate(const float* in, float* out, int64_t n, cudaStream_t s) {
    if (n == 0) return;
    negate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, out, n);
    LB_LAUNCH();
}

__global__ void restore_alpha_kernel(RowMap rows, const int* __restrict__ first_save,
                                     const int* __restrict__ keep_current, int n,
                                     const float* __restrict__ best, float* __restrict__ alpha) {
    for (int r2 = blockIdx.y; r2 < 2 * rows.R; r2 += gridDim.y) {
        const int rr = r2 >= rows.R ? r2 - rows.R : r2;
        const int bx = rows.row_box[rr];
        if (!first_save[bx] && !(keep_current && keep_current[bx]))
            copy_row(best + (size_t)r2 * n, alpha + (size_t)r2 * n, n);
    }
}

void launch_restore_alpha(const RowMap& rows, const int* first_save, int n, const float* best_alpha,
                          float* alpha, cudaStream_t s, const int* keep_current) {
    if (rows.R == 0 || n == 0) return;
    const dim3 grid(ceil_div(n, 1024), std::min(2 * rows.R, 65535));
    restore_alpha_kernel<<<grid, 256, 0, s>>>(rows, first_save, keep_current, n, best_alpha, alpha);
    LB_LAUNCH();
}

// ---- warm start ---------------------------------------------------------------
__global__ void warm_seed_kernel(const int* __restrict__ box_off, const int* __restrict__ prev_box_off,
                                 const int* __restrict__ parent, int B, int* __restrict__ seed) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int p = parent[b];
    seed[b] = (p >= 0 && box_off[b + 1] - box_off[b] == prev_box_off[p + 1] - prev_box_off[p]) ? 1 : 0;
}

void launch_warm_seed(const int* box_off, const int* prev_box_off, const int* parent, int B, int* seed,
                      cudaStream_t s) {
    if (B == 0) return;
    warm_seed_kernel<<<ceil_div(B, 256), 256, 0, s>>>(box_off, prev_box_off, parent, B, seed);
    LB_LAUNCH();
}

__global__ void warm_alpha_kernel(RowMap rows, const int* __restrict__ seed, const int* __restrict__ parent,
                                  const int* __restrict__ prev_box_off, int prev_R, int n,
                                  const float* __restrict__ prev_alpha, float* __restrict__ alpha) {
    for (int r2 = blockIdx.y; r2 < 2 * rows.R; r2 += gridDim.y) {
        const int side = r2 >= rows.R ? 1 : 0;
        const int rr = r2 - side * rows.R;
        const int bx = rows.row_box[rr];
        if (!seed[bx]) continue;
        const int src = side * prev_R + prev_box_off[parent[bx]] + (rr - rows.box_off[bx]);
        copy_row(prev_alpha + (size_t)src * n, alpha + (size_t)r2 * n, n);
    }
}

void launch_warm_alpha(const RowMap& rows, const int* seed, const int* parent, const int* prev_box_off, int prev_R,
                       int n, const float* prev_alpha, float* alpha, cudaStream_t s) {
    if (rows.R == 0 || n == 0) return;
    const dim3 grid(ceil_div(n, 1024), std::min(2 * rows.R, 65535));
    warm_alpha_kernel<<<grid, 256, 0, s>>>(rows, seed, parent, prev_box_off, prev_R, n, prev_alpha, alpha);
    LB_LAUNCH();
}

// One block per box: the creation set a start uses (the parent's for a
// seeded box, the box's own otherwise) and whether it is non-empty.
__global__ void warm_aset_kernel(const int* __restrict__ seed, const int* __restrict__ parent, int n,
                                 const uint8_t* __restrict__ prev_aset, const uint8_t* __restrict__ aset,
                                 uint8_t* __restrict__ out, int* __restrict__ has) {
    const int b = blockIdx.x;
    const uint8_t* src = seed[b] ? prev_aset + (size_t)parent[b] * n : aset + (size_t)b * n;
    int any = 0;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const uint8_t v = src[j];
        out[(size_t)b * n + j] = v;
        any |= v;
    }
    any = __syncthreads_or(any);
    if (threadIdx.x == 0) has[b] = any ? 1 : 0;
}

void launch_warm_aset(const int* seed, const int* parent, int B, int n, const uint8_t* prev_aset,
                      const uint8_t* aset, uint8_t* out, int* has, cudaStream_t s) {
    if (B == 0) return;
    warm_aset_kernel<<<B, 256, 0, s>>>(seed, parent, n, prev_aset, aset, out, has);
    LB_LAUNCH();
}

__global__ void ibp_spec_kernel(const float* __restrict__ C, int c_per_box, const float* __restrict__ l,
                                const float* __restrict__ u, int B, int nspec, int nout,
                                float* __restrict__ lb, float* __restrict__ ub) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * nspec) return;
    const int bx = i / nspec, j = i % nspec;
    const float* c = C + ((size_t)(c_per_box ? bx : 0) * nspec + j) * nout;
    const float* lv = l + (size_t)bx * nout;
    const float* uv = u + (size_t)bx * nout;
    float lp = 0.f, ln = 0.f, up = 0.f, un = 0.f;
    for (int k = 0; k < nout; ++k) {
        const float cp = fmaxf(c[k], 0.f), cn = fminf(c[k], 0.f);
        lp = fmaf(cp, lv[k], lp);
        ln = fmaf(cn, uv[k], ln);
        up = fmaf(cp, uv[k], up);
        un = fmaf(cn, lv[k], un);
    }
    lb[i] = lp + ln;
    ub[i] = up + un;
}

void launch_ibp_spec(const float* C, int c_per_box, const float* l, const float* u, int B, int nspec,
                     int nout, float* lb, float* ub, cudaStream_t s) {
    if (B * nspec == 0) return;
    ibp_spec_kernel<<<ceil_div(B * nspec, 128), 128, 0, s>>>(C, c_per_box, l, u, B, nspec, nout, lb, ub);
    LB_LAUNCH();
}

__global__ void input_sub_kernel(const float* __restrict__ c, bool neg, const float* __restrict__ xl,
                                 const float* __restrict__ xu, float* __restrict__ ol, float* __restrict__ ou,
                                 int64_t total, int n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const float k = c[i % n];
    if (neg) {
        ol[i] = k - xu[i];
        ou[i] = k - xl[i];
    } else {
        ol[i] = xl[i] - k;
        ou[i] = xu[i] - k;
    }
}

void launch_input_sub(const float* c, bool neg, const float* xl, const float* xu, float* ol, float* ou, int B, int n,
                      cudaStream_t s) {
    const int64_t total = (int64_t)B * n;
    if (total == 0) return;
    input_sub_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(c, neg, xl, xu, ol, ou, total, n);
    LB_LAUNCH();
}

__global__ void add_bounds_kernel(float* __restrict__ ol, float* __restrict__ ou, const float* __restrict__ il,
                                  const float* __restrict__ iu, int64_t n, bool relu_in) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float l = relu_in ? fmaxf(il[i], 0.f) : il[i];
    const float u = relu_in ? fmaxf(iu[i], 0.f) : iu[i];
    ol[i] += l;
    ou[i] += u;
}

void launch_add_bounds(float* out_l, float* out_u, const float* in_l, const float* in_u, int64_t n, bool relu_in,
                       cudaStream_t s) {
    if (n == 0) return;
    add_bounds_kernel<<<ceil_div(n, 256), 256, 0, s>>>(out_l, out_u, in_l, in_u, n, relu_in);
    LB_LAUNCH();
}

// ============================================================== Sigmoid
namespace {
__device__ __forceinline__ float sig_f(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float dsig_f(float x) {
    const float s = sig_f(x);
    return s * (1.f - s);
}
__device__ __forceinline__ float d2sig_f(float x) {
    const float s = sig_f(x);
    return s * (1.f - s) * (1.f - 2.f * s);
}
constexpr float SIG_STEP = 0.01f;

// Tangent point whose tangent passes through (b, sigmoid(b)) from below
// (table d_lower at b = 0.01 i) or from above (table d_upper at b = -0.01 i).
__device__ float sig_table_point(int i, bool lower_table) {
    const float b = lower_table ? SIG_STEP * (float)i : -SIG_STEP * (float)i;
    const float yb = sig_f(b);
    auto ok = [&](float d) {
        const float v = dsig_f(d) * (b - d) + sig_f(d);
        return lower_table ? v <= yb : v >= yb;
    };
    if (lower_table) {
        float l = -1.f, r = 0.f;
        for (int t = 0; t < 64 && !ok(l); ++t) l *= 2.f;
        for (int t = 0; t < 100; ++t) {
            const float m = (l + r) / 2.f;
            if (ok(m)) l = m;
            else r = m;
        }
        return l;
    }
    float l = 0.f, r = 1.f;
    for (int t = 0; t < 64 && !ok(r); ++t) r *= 2.f;
    for (int t = 0; t < 100; ++t) {
        const float m = (l + r) / 2.f;
        if (ok(m)) r = m;
        else l = m;
    }
    return r;
}

__device__ __forceinline__ int sig_index(float b) {
    const float q = b / SIG_STEP;
    return (q > 0.f ? (int)q : 0) + 1;  // max(0, trunc(q)) + 1
}

struct SigLines {
    float kd;           // secant slope (or sigmoid'(l) for a tiny interval)
    bool pos, neg, both, mdl, mdu, same;
};

__device__ __forceinline__ SigLines sig_cases(float l, float u) {
    SigLines c;
    c.pos = l >= 0.f;
    c.neg = u <= 0.f;
    c.both = !(c.pos || c.neg);
    const float yl = sig_f(l), yu = sig_f(u);
    c.same = fabsf(u - l) < 1e-4f;
    c.kd = c.same ? dsig_f(l) : (yu - yl) / fmaxf(u - l, 1e-8f);
    c.mdl = c.both && c.kd < dsig_f(l);
    c.mdu = c.both && c.kd < dsig_f(u);
    return c;
}
}  // namespace

__global__ void sigmoid_params_kernel(const float* __restrict__ l, const float* __restrict__ u, int64_t total,
                                      float* __restrict__ lw, float* __restrict__ lb, float* __restrict__ uw,
                                      float* __restrict__ ub, uint8_t* __restrict__ flags) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const float lv = l[i], uv = u[i];
    const SigLines c = sig_cases(lv, uv);
    const float yl = sig_f(lv);
    const float sec_b = yl - c.kd * lv;
    const float m = (lv + uv) / 2.f;
    const float km = dsig_f(m), bm = sig_f(m) - km * m;
    float wl, bl, wu, bu;
    if (c.pos) {
        wl = c.kd, bl = sec_b, wu = km, bu = bm;
    } else if (c.neg) {
        wl = km, bl = bm, wu = c.kd, bu = sec_b;
    } else {
        if (c.mdl) {
            wl = c.kd, bl = sec_b;
        } else {
            const float d = sig_table_point(sig_index(uv), true);
            wl = dsig_f(d);
            bl = sig_f(d) - wl * d;
        }
        if (c.mdu) {
            wu = c.kd, bu = sec_b;
        } else {
            const float d = sig_table_point(sig_index(-lv), false);
            wu = dsig_f(d);
            bu = sig_f(d) - wu * d;
        }
    }
    lw[i] = wl;
    lb[i] = bl;
    uw[i] = wu;
    ub[i] = bu;
    flags[i] = RF_UNSTABLE;
}

void launch_sigmoid_params(const float* l, const float* u, int B, int n, float* lw, float* lb, float* uw, float* ub,
                           uint8_t* flags, cudaStream_t s) {
    const int64_t total = (int64_t)B * n;
    if (total == 0) return;
    sigmoid_params_kernel<<<ceil_div(total, 128), 128, 0, s>>>(l, u, total, lw, lb, uw, ub, flags);
    LB_LAUNCH();
}

__global__ void sigmoid_bound_grad_kernel(RowMap rows, const float* __restrict__ cur_l,
                                          const float* __restrict__ cur_u, const float* __restrict__ sbar,
                                          const float* __restrict__ blbar, const float* __restrict__ kbar,
                                          const float* __restrict__ bbar, int n, float* __restrict__ g) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows.R) return;
    const size_t at = (size_t)rows.row_box[r] * n + rows.row_id[r];
    const float l = cur_l[at], u = cur_u[at];
    const SigLines c = sig_cases(l, u);
    // Secant line (k = kd, b = sigmoid(l) - kd l) and midpoint tangent
    // (k = sigmoid'(m), b = sigmoid(m) - k m, m = (l + u) / 2).
    float dkd_dl, dkd_du;
    if (c.same) {
        dkd_dl = d2sig_f(l);
        dkd_du = 0.f;
    } else {
        const float D = fmaxf(u - l, 1e-8f), dy = sig_f(u) - sig_f(l);
        dkd_du = dsig_f(u) / D - dy / (D * D);
        dkd_dl = -dsig_f(l) / D + dy / (D * D);
    }
    float gl = 0.f, gu = 0.f;
    auto secant = [&](float wb, float bb) {
        const float t = wb - l * bb;
        gl += t * dkd_dl + bb * (dsig_f(l) - c.kd);
        gu += t * dkd_du;
    };
    auto midpoint = [&](float wb, float bb) {
        const float m = (l + u) / 2.f;
        const float gm = d2sig_f(m) * (wb - m * bb);
        gl += 0.5f * gm;
        gu += 0.5f * gm;
    };
    const float sb = sbar[at], lbb = blbar[at], kb = kbar[at], bb = bbar[at];
    if (c.pos) {
        secant(sb, lbb);
        midpoint(kb, bb);
    } else if (c.neg) {
        midpoint(sb, lbb);
        secant(kb, bb);
    } else {
        if (c.mdl) secant(sb, lbb);
        if (c.mdu) secant(kb, bb);
    }
    g[r] = gl;
    g[rows.R + r] = gu;
}

void launch_sigmoid_bound_grad(const RowMap& rows, const float* cur_l, const float* cur_u, const float* sbar,
                               const float* blbar, const float* kbar, const float* bbar, int n, float* g,
                               cudaStream_t s) {
    if (rows.R == 0) return;
    sigmoid_bound_grad_kernel<<<ceil_div(rows.R, 256), 256, 0, s>>>(rows, cur_l, cur_u, sbar, blbar, kbar, bbar, n,
                                                                    g);
    LB_LAUNCH();
}

__global__ void sigmoid_bounds_kernel(const float* __restrict__ l, const float* __restrict__ u, float* __restrict__ ol,
                                      float* __restrict__ ou, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    ol[i] = sig_f(l[i]);
    ou[i] = sig_f(u[i]);
}

void launch_sigmoid_bounds(const float* l, const float* u, float* ol, float* ou, int64_t n, cudaStream_t s) {
    if (n == 0) return;
    sigmoid_bounds_kernel<<<ceil_div(n, 256), 256, 0, s>>>(l, u, ol, ou, n);
    LB_LAUNCH();
}

// ============================================================== helpers
__global__ void fill_f32_kernel(float* p, float v, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

void launch_fill_f32(float* p, float v, int64_t n, cudaStream_t s) {
    if (n == 0) return;
    fill_f32_kernel<<<ceil_div(n, 256), 256, 0, s>>>(p, v, n);
    LB_LAUNCH();
}

__global__ void expand_spec_kernel(const float* C, int c_per_box, int B, int per, float* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * per) return;
    const int bx = (int)(i / per), k = (int)(i % per);
    out[i] = C[(size_t)(c_per_box ? bx : 0) * per + k];
}

void launch_expand_spec(const float* C, int c_per_box, int B, int nspec, int nout, float* out,
                        cudaStream_t s) {
    const int per = nspec * nout;
    expand_spec_kernel<<<ceil_div((int64_t)B * per, 256), 256, 0, s>>>(C, c_per_box, B, per, out);
    LB_LAUNCH();
}

}  // namespace lb200
