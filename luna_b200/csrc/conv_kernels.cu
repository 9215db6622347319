// conv_kernels.cu -- SIMT kernels of the conv layers (IBP, windowed
// transposed-conv steps with fused relaxation / concretisation, and their
// adjoints).
#include "conv_kernels.cuh"

#include <algorithm>
#include <stdexcept>

namespace lb200 {

namespace {

__device__ __forceinline__ void row_split(int r, int R, int& p, int& rr) {
    p = r >= R ? 1 : 0;
    rr = r - p * R;
}

__device__ __forceinline__ void win_origin(const WinGeo& g, int row_id, int& oy, int& ox) {
    if (g.full) {
        oy = 0;
        ox = 0;
        return;
    }
    const int pix = row_id / g.st_C;
    const int y0 = pix / g.st_W, x0 = pix - (pix / g.st_W) * g.st_W;
    oy = g.mul_y * y0 + g.off_y;
    ox = g.mul_x * x0 + g.off_x;
}

// Map neuron of window element j of a row whose window starts at (oy, ox),
// or -1 outside the map.
__device__ __forceinline__ int win_neuron(const WinGeo& g, int oy, int ox, int j) {
    if (g.full) return j;
    const int c = j % g.C, pix = j / g.C;
    const int wy = pix / g.ww, wx = pix - wy * g.ww;
    const int y = oy + wy, x = ox + wx;
    if ((unsigned)y >= (unsigned)g.H || (unsigned)x >= (unsigned)g.W) return -1;
    return (y * g.W + x) * g.C + c;
}

// Lower side: Q = P+ s + P- k, bias P- b; upper side: Q = P+ k + P- s, bias
// P+ b (BoundedReLUNode.cpp:179-195,268-285).
__device__ __forceinline__ float relax_q(float P, int p, float s, float k, float b, float& bias) {
    const float pos = fmaxf(P, 0.f), neg = fminf(P, 0.f);
    if (p == 0) {
        bias += neg * b;
        return pos * s + neg * k;
    }
    bias += pos * b;
    return pos * k + neg * s;
}

// Block-wide sum (blockDim.x == 256) returned to thread 0.
__device__ __forceinline__ float block_sum256(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x == 0)
        for (int w = 0; w < 8; ++w) t += sh[w];
    return t;
}

// One element of the transposed convolution of one row's window.
__device__ __forceinline__ float convT_elem(const float* __restrict__ Arow, const ConvStep& cs, int j) {
    const int ci = j % cs.Ci, pix = j / cs.Ci;
    const int vy = pix / cs.out_w, vx = pix - vy * cs.out_w;
    const int ty = vy + cs.cy, tx = vx + cs.cx;
    float acc = 0.f;
    for (int ky = ty % cs.sh; ky < cs.kh && ky <= ty; ky += cs.sh) {
        const int qy = (ty - ky) / cs.sh;
        if (qy >= cs.in_h) continue;
        for (int kx = tx % cs.sw; kx < cs.kw && kx <= tx; kx += cs.sw) {
            const int qx = (tx - kx) / cs.sw;
            if (qx >= cs.in_w) continue;
            const float* a = Arow + ((size_t)qy * cs.in_w + qx) * cs.Co;
            const float* w = cs.Wk + ((size_t)(ky * cs.kw + kx) * cs.Co) * cs.Ci + ci;
            for (int co = 0; co < cs.Co; ++co) acc = fmaf(a[co], w[(size_t)co * cs.Ci], acc);
        }
    }
    return acc;
}

}  // namespace

// ============================================================== IBP
__global__ void ibp_conv_kernel(const float* __restrict__ Wc, const float* __restrict__ bias,
                                const float* __restrict__ in_l, const float* __restrict__ in_u,
                                float* __restrict__ out_l, float* __restrict__ out_u, int B, int Ci, int Hi,
                                int Wi, int Co, int Ho, int Wo, int kh, int kw, int sh, int sw, int ph, int pw,
                                bool relu_in) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)B * Ho * Wo * Co;
    if (idx >= total) return;
    const int co = (int)(idx % Co);
    int64_t t = idx / Co;
    const int xo = (int)(t % Wo);
    t /= Wo;
    const int yo = (int)(t % Ho);
    const int bx = (int)(t / Ho);
    float lp = 0.f, ln = 0.f, up = 0.f, un = 0.f;
    for (int ky = 0; ky < kh; ++ky) {
        const int yi = yo * sh - ph + ky;
        if (yi < 0 || yi >= Hi) continue;
        for (int kx = 0; kx < kw; ++kx) {
            const int xi = xo * sw - pw + kx;
            if (xi < 0 || xi >= Wi) continue;
            const float* w = Wc + ((size_t)(co * kh + ky) * kw + kx) * Ci;
            const size_t base = (((size_t)bx * Hi + yi) * Wi + xi) * Ci;
            for (int ci = 0; ci < Ci; ++ci) {
                float l = in_l[base + ci], u = in_u[base + ci];
                if (relu_in) {
                    l = fmaxf(l, 0.f);
                    u = fmaxf(u, 0.f);
                }
                const float wv = w[ci];
                if (wv >= 0.f) {
                    lp = fmaf(wv, l, lp);
                    up = fmaf(wv, u, up);
                } else {
                    ln = fmaf(wv, u, ln);
                    un = fmaf(wv, l, un);
                }
            }
        }
    }
    const float b = bias ? bias[co] : 0.f;
    out_l[idx] = (lp + ln) + b;
    out_u[idx] = (up + un) + b;
}

void launch_ibp_conv(const float* Wc, const float* b, const float* in_l, const float* in_u, float* out_l,
                     float* out_u, int B, int Ci, int Hi, int Wi, int Co, int Ho, int Wo, int kh, int kw,
                     int sh, int sw, int ph, int pw, bool relu_in, cudaStream_t s) {
    const int64_t total = (int64_t)B * Ho * Wo * Co;
    if (total == 0) return;
    ibp_conv_kernel<<<ceil_div(total, 256), 256, 0, s>>>(Wc, b, in_l, in_u, out_l, out_u, B, Ci, Hi, Wi, Co,
                                                         Ho, Wo, kh, kw, sh, sw, ph, pw, relu_in);
    LB_LAUNCH();
}

__global__ void chw_to_hwc_kernel(const float* __restrict__ src, float* __restrict__ dst, int B, int C, int H,
                                  int W) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = (int64_t)C * H * W;
    if (idx >= (int64_t)B * n) return;
    const int64_t bx = idx / n;
    const int i = (int)(idx - bx * n);  // HWC index
    const int c = i % C, pix = i / C;
    dst[idx] = src[bx * n + (int64_t)c * H * W + pix];
}

void launch_chw_to_hwc(const float* src, float* dst, int B, int C, int H, int W, cudaStream_t s) {
    const int64_t total = (int64_t)B * C * H * W;
    if (total == 0) return;
    chw_to_hwc_kernel<<<ceil_div(total, 256), 256, 0, s>>>(src, dst, B, C, H, W);
    LB_LAUNCH();
}

// One warp per box; neurons visited in CHW order.
__global__ void fill_rows_chw_kernel(const float* __restrict__ l, const float* __restrict__ u, int B, int C,
                                     int H, int W, const int* __restrict__ off, int* __restrict__ row_box,
                                     int* __restrict__ row_id) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= B) return;
    const int HW = H * W, n = C * HW;
    int base = off[warp];
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        bool un = false;
        int sidx = 0;
        if (i < n) {
            const int c = i / HW, pix = i - c * HW;
            sidx = pix * C + c;
            const float lv = l[(size_t)warp * n + sidx], uv = u[(size_t)warp * n + sidx];
            un = lv < 0.f && uv > 0.f;
        }
        const unsigned m = __ballot_sync(0xffffffffu, un);
        if (un) {
            const int pos = base + __popc(m & ((1u << lane) - 1u));
            row_box[pos] = warp;
            row_id[pos] = sidx;
        }
        base += __popc(m);
    }
}

void launch_fill_rows_chw(const float* l, const float* u, int B, int C, int H, int W, const int* box_off,
                          int* row_box, int* row_id, cudaStream_t s) {
    fill_rows_chw_kernel<<<ceil_div((int64_t)B * 32, 256), 256, 0, s>>>(l, u, B, C, H, W, box_off, row_box,
                                                                        row_id);
    LB_LAUNCH();
}

// ============================================================== start step
__global__ void __launch_bounds__(256) conv_start_step_kernel(ConvStartStep st) {
    __shared__ float sh[8];
    const int r = blockIdx.x;
    int p, rr;
    row_split(r, st.rows.R, p, rr);
    const int bx = st.rows.row_box[rr];
    const int id = st.rows.row_id[rr];
    const bool whole = st.g.full != 0;
    const WinGeo& wgeo = whole ? st.wg : st.g;  // the weight window's geometry
    const int co = id % wgeo.st_C;
    const int nwin = wgeo.size();
    const int nw = st.g.size();
    int oy, ox;
    win_origin(st.g, id, oy, ox);
    int wy0 = 0, wx0 = 0;
    if (whole) win_origin(wgeo, id, wy0, wx0);
    const float* wrow = st.Wc + (size_t)co * nwin;
    float part = 0.f;
    for (int j = threadIdx.x; j < nw; j += blockDim.x) {
        float P;
        if (whole) {
            // Map element j -> weight window element, or 0 outside it.
            const int c = j % st.g.C, pix = j / st.g.C;
            const int wy = pix / st.g.W - wy0, wx = pix - (pix / st.g.W) * st.g.W - wx0;
            P = ((unsigned)wy < (unsigned)wgeo.wh && (unsigned)wx < (unsigned)wgeo.ww)
                    ? wrow[(wy * wgeo.ww + wx) * wgeo.C + c]
                    : 0.f;
        } else {
            P = wrow[j];
        }
        const size_t at = (size_t)r * nw + j;
        if (st.P_save) st.P_save[at] = P;
        const int nu = win_neuron(st.g, oy, ox, j);
        float Q = 0.f;
        if (nu >= 0) {
            const size_t bj = (size_t)bx * st.rp.n + nu;
            const float s = (st.alpha && (st.rp.flags[bj] & RF_USE_ALPHA)) ? st.alpha[at] : st.rp.slope_lo[bj];
            Q = relax_q(P, p, s, st.rp.k_up[bj], st.rp.b_up[bj], part);
            if (st.b_next) part = fmaf(Q, st.b_next[j % st.g.C], part);
        }
        st.Q[at] = Q;
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) st.bias_acc[r] = st.bW[co] + tot;
}

void launch_conv_start_step(const ConvStartStep& st, cudaStream_t s) {
    if (st.M == 0) return;
    conv_start_step_kernel<<<st.M, 256, 0, s>>>(st);
    LB_LAUNCH();
}

// ============================================================== convT steps
int conv_chunks(const WinGeo& out) { return ceil_div(out.size(), 256); }

__global__ void __launch_bounds__(256) convT_relax_kernel(const float* __restrict__ A, ConvStep cs, int M,
                                                          ConvRelaxEpi e, int nchunk, float* __restrict__ partial) {
    __shared__ float sh[8];
    const int r = (int)(blockIdx.x / nchunk), chunk = (int)(blockIdx.x % nchunk);
    const int nin = cs.in_h * cs.in_w * cs.Co;
    const int nw = e.g.size();
    const int j = chunk * 256 + threadIdx.x;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    float part = 0.f;
    if (j < nw) {
        const size_t at = (size_t)r * nw + j;
        float P = convT_elem(A + (size_t)r * nin, cs, j);
        if (e.addend) P += e.addend[at];
        if (e.P_save) e.P_save[at] = P;
        int oy, ox;
        win_origin(e.g, e.rows.row_id[rr], oy, ox);
        const int nu = win_neuron(e.g, oy, ox, j);
        float Q = 0.f;
        if (nu >= 0) {
            const size_t bj = (size_t)bx * e.rp.n + nu;
            const float s = (e.alpha && (e.rp.flags[bj] & RF_USE_ALPHA)) ? e.alpha[at] : e.rp.slope_lo[bj];
            Q = relax_q(P, p, s, e.rp.k_up[bj], e.rp.b_up[bj], part);
            if (e.b_next) part = fmaf(Q, e.b_next[j % e.g.C], part);
        }
        e.Q[at] = Q;
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) partial[(size_t)chunk * M + r] = tot;
}

__global__ void __launch_bounds__(256) convT_conc_kernel(const float* __restrict__ A, ConvStep cs, int M,
                                                         ConvConcEpi e, int nchunk, float* __restrict__ partial) {
    __shared__ float sh[8];
    const int r = (int)(blockIdx.x / nchunk), chunk = (int)(blockIdx.x % nchunk);
    const int nin = cs.in_h * cs.in_w * cs.Co;
    const int nw = e.g.size();
    const int n0 = e.g.C * e.g.H * e.g.W;
    const int j = chunk * 256 + threadIdx.x;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    float part = 0.f;
    if (j < nw) {
        const float P = convT_elem(A + (size_t)r * nin, cs, j);
        int oy, ox;
        win_origin(e.g, e.rows.row_id[rr], oy, ox);
        const int nu = win_neuron(e.g, oy, ox, j);
        uint8_t sg = 0;
        if (nu >= 0) {
            const float xl = e.xl[(size_t)bx * n0 + nu], xu = e.xu[(size_t)bx * n0 + nu];
            if (e.form == CONC_PATCHES) {
                const float c = (xu + xl) / 2.0f, d = (xu - xl) / 2.0f;
                part = p == 0 ? fmaf(P, c, -fabsf(P) * d) : fmaf(P, c, fabsf(P) * d);
                sg = (uint8_t)((P > 0.f ? 1 : 0) | (P < 0.f ? 2 : 0));
            } else {
                const float xa = p == 0 ? xl : xu, xb = p == 0 ? xu : xl;
                part = fmaxf(P, 0.f) * xa + fminf(P, 0.f) * xb;
                sg = (uint8_t)((P >= 0.f ? 1 : 0) | (P <= 0.f ? 2 : 0));
            }
        }
        if (e.sign) e.sign[(size_t)r * nw + j] = sg;
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) partial[(size_t)chunk * M + r] = tot;
}

void launch_convT_relax(const float* A, const ConvStep& cs, int M, const ConvRelaxEpi& e, float* partial,
                        cudaStream_t s) {
    if (M == 0) return;
    const int nchunk = conv_chunks(e.g);
    convT_relax_kernel<<<(unsigned)((int64_t)M * nchunk), 256, 0, s>>>(A, cs, M, e, nchunk, partial);
    LB_LAUNCH();
}

void launch_convT_conc(const float* A, const ConvStep& cs, int M, const ConvConcEpi& e, float* partial,
                       cudaStream_t s) {
    if (M == 0) return;
    const int nchunk = conv_chunks(e.g);
    convT_conc_kernel<<<(unsigned)((int64_t)M * nchunk), 256, 0, s>>>(A, cs, M, e, nchunk, partial);
    LB_LAUNCH();
}

// ============================================================== register-blocked steps
constexpr int RB_MAX_W_FLOATS = 12 * 1024;  // 48 KB of weights in shared memory

bool convT_rb_ok(const ConvStep& cs) {
    return (cs.Ci == 8 || cs.Ci == 16 || cs.Ci == 32) && cs.Co % 4 == 0 && cs.cy >= 0 && cs.cx >= 0 &&
           (int64_t)cs.kh * cs.kw * cs.Co * cs.Ci <= RB_MAX_W_FLOATS;
}

int convT_rb_chunks(const WinGeo& out) { return ceil_div(out.wh * out.ww, 256); }

// Work items: with gs == 256, one 256-pixel chunk of one row (nchunk per
// row, block-wide partial sum); with gs a power of two <= 32 (windows of at
// most gs pixels), 256 / gs rows per item, one gs-lane group per row
// (shuffle partial sum).  Blocks are persistent over the items, so the
// layer's weights are staged in shared memory once per block.
template <int CI>
__global__ void __launch_bounds__(256, CI <= 16 ? 3 : 2) convT_relax_rb_kernel(const float* __restrict__ A, ConvStep cs, int M,
                                                             ConvRelaxEpi e, int nchunk, int gs,
                                                             float* __restrict__ partial) {
    extern __shared__ float4 rb_w4[];
    float* wsh = reinterpret_cast<float*>(rb_w4);
    __shared__ float red[8];
    const int nwt = cs.kh * cs.kw * cs.Co * CI;
    for (int i = threadIdx.x; i < nwt; i += blockDim.x) wsh[i] = cs.Wk[i];
    __syncthreads();
    const int npix = cs.out_h * cs.out_w;
    const int rpb = 256 / gs;
    const int64_t items = gs == 256 ? (int64_t)M * nchunk : ((int64_t)M + rpb - 1) / rpb;
    for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    int r, chunk, pix;
    if (gs == 256) {
        r = (int)(w / nchunk);
        chunk = (int)(w - (int64_t)r * nchunk);
        pix = chunk * 256 + threadIdx.x;
    } else {
        r = (int)(w * rpb) + (int)threadIdx.x / gs;
        chunk = 0;
        pix = (int)threadIdx.x % gs;
    }
    float part = 0.f;
    if (r < M && pix < npix) {
        int p, rr;
        row_split(r, e.rows.R, p, rr);
        const int bx = e.rows.row_box[rr];
        float acc[CI];
#pragma unroll
        for (int c = 0; c < CI; ++c) acc[c] = 0.f;
        const int vy = pix / cs.out_w, vx = pix - (pix / cs.out_w) * cs.out_w;
        const int ty = vy + cs.cy, tx = vx + cs.cx;
        const float* Arow = A + (size_t)r * cs.in_h * cs.in_w * cs.Co;
        for (int ky = ty % cs.sh; ky < cs.kh && ky <= ty; ky += cs.sh) {
            const int qy = (ty - ky) / cs.sh;
            if (qy >= cs.in_h) continue;
            for (int kx = tx % cs.sw; kx < cs.kw && kx <= tx; kx += cs.sw) {
                const int qx = (tx - kx) / cs.sw;
                if (qx >= cs.in_w) continue;
                const float4* a4 = reinterpret_cast<const float4*>(Arow + ((size_t)qy * cs.in_w + qx) * cs.Co);
                const float* wt = wsh + (size_t)(ky * cs.kw + kx) * cs.Co * CI;
                for (int c4 = 0; c4 < cs.Co / 4; ++c4) {
                    const float4 a = __ldg(a4 + c4);
                    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float4* wr = reinterpret_cast<const float4*>(wt + (size_t)(c4 * 4 + t) * CI);
#pragma unroll
                        for (int c = 0; c < CI / 4; ++c) {
                            const float4 wv = wr[c];
                            acc[4 * c + 0] = fmaf(av[t], wv.x, acc[4 * c + 0]);
                            acc[4 * c + 1] = fmaf(av[t], wv.y, acc[4 * c + 1]);
                            acc[4 * c + 2] = fmaf(av[t], wv.z, acc[4 * c + 2]);
                            acc[4 * c + 3] = fmaf(av[t], wv.w, acc[4 * c + 3]);
                        }
                    }
                }
            }
        }
        const size_t at0 = (size_t)r * npix * CI + (size_t)pix * CI;
        int oy, ox;
        win_origin(e.g, e.rows.row_id[rr], oy, ox);
        const int nu0 = win_neuron(e.g, oy, ox, pix * CI);  // the pixel's channel 0, or -1 outside the map
#pragma unroll
        for (int c = 0; c < CI; c += 4) {
            float Pv[4] = {acc[c], acc[c + 1], acc[c + 2], acc[c + 3]};
            if (e.addend) {
                const float4 ad = *reinterpret_cast<const float4*>(e.addend + at0 + c);
                Pv[0] += ad.x;
                Pv[1] += ad.y;
                Pv[2] += ad.z;
                Pv[3] += ad.w;
            }
            if (e.P_save) *reinterpret_cast<float4*>(e.P_save + at0 + c) = make_float4(Pv[0], Pv[1], Pv[2], Pv[3]);
            float Qv[4] = {0.f, 0.f, 0.f, 0.f};
            if (nu0 >= 0) {
                const size_t bj = (size_t)bx * e.rp.n + nu0 + c;
                const float4 s4 = *reinterpret_cast<const float4*>(e.rp.slope_lo + bj);
                const float4 k4 = *reinterpret_cast<const float4*>(e.rp.k_up + bj);
                const float4 b4 = *reinterpret_cast<const float4*>(e.rp.b_up + bj);
                const uchar4 f4 = *reinterpret_cast<const uchar4*>(e.rp.flags + bj);
                float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (e.alpha && ((f4.x | f4.y | f4.z | f4.w) & RF_USE_ALPHA))
                    a4 = *reinterpret_cast<const float4*>(e.alpha + at0 + c);
                const float Av[4] = {a4.x, a4.y, a4.z, a4.w};
                const float sl[4] = {s4.x, s4.y, s4.z, s4.w}, ku[4] = {k4.x, k4.y, k4.z, k4.w},
                            bu[4] = {b4.x, b4.y, b4.z, b4.w};
                const uint8_t fl[4] = {f4.x, f4.y, f4.z, f4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float sv = (e.alpha && (fl[i] & RF_USE_ALPHA)) ? Av[i] : sl[i];
                    Qv[i] = relax_q(Pv[i], p, sv, ku[i], bu[i], part);
                    if (e.b_next) part = fmaf(Qv[i], e.b_next[c + i], part);
                }
            }
            *reinterpret_cast<float4*>(e.Q + at0 + c) = make_float4(Qv[0], Qv[1], Qv[2], Qv[3]);
        }
    }
    if (gs == 256) {
        const float tot = block_sum256(part, red);
        if (threadIdx.x == 0) partial[(size_t)chunk * M + r] = tot;
        __syncthreads();  // red[] is reused by the next item
    } else {
        for (int o = gs >> 1; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((int)threadIdx.x % gs == 0 && r < M) partial[r] = part;
    }
    }
}

// Resident blocks of a kernel with `smem` dynamic shared memory, times 148-SM
// waves: the grid of the persistent register-blocked conv kernels.
template <class K>
int rb_grid(K kernel, size_t smem, int64_t items) {
    int per_sm = 1, dev = 0, sms = 148;
    LB_CUDA(cudaGetDevice(&dev));
    LB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    LB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem));
    return (int)std::max<int64_t>(1, std::min<int64_t>(items, (int64_t)std::max(per_sm, 1) * sms * 4));
}

void launch_convT_relax_rb(const float* A, const ConvStep& cs, int M, const ConvRelaxEpi& e, float* partial,
                           cudaStream_t s) {
    if (M == 0) return;
    if (!convT_rb_ok(cs) || e.g.C != cs.Ci || e.g.wh != cs.out_h || e.g.ww != cs.out_w)
        throw std::invalid_argument("convT_relax_rb: unsupported step");
    const int nchunk = convT_rb_chunks(e.g);
    const size_t smem = (size_t)cs.kh * cs.kw * cs.Co * cs.Ci * 4;
    // Windows of at most 32 pixels: several rows per work item.
    const int npix = cs.out_h * cs.out_w;
    int gs = 256;
    if (npix <= 32) {
        gs = 1;
        while (gs < npix) gs <<= 1;
    }
    const int64_t items = gs == 256 ? (int64_t)M * nchunk : ((int64_t)M + 256 / gs - 1) / (256 / gs);
    if (cs.Ci == 8) {
        const int grid = rb_grid(convT_relax_rb_kernel<8>, smem, items);
        convT_relax_rb_kernel<8><<<grid, 256, smem, s>>>(A, cs, M, e, nchunk, gs, partial);
    } else if (cs.Ci == 16) {
        const int grid = rb_grid(convT_relax_rb_kernel<16>, smem, items);
        convT_relax_rb_kernel<16><<<grid, 256, smem, s>>>(A, cs, M, e, nchunk, gs, partial);
    } else {
        const int grid = rb_grid(convT_relax_rb_kernel<32>, smem, items);
        convT_relax_rb_kernel<32><<<grid, 256, smem, s>>>(A, cs, M, e, nchunk, gs, partial);
    }
    LB_LAUNCH();
}

bool conv_adj_rb_ok(const ConvStep& cs) {
    return (cs.Co == 8 || cs.Co == 16 || cs.Co == 32) && cs.Ci % 4 == 0 &&
           (int64_t)cs.kh * cs.kw * cs.Co * cs.Ci <= RB_MAX_W_FLOATS;
}

template <int CO>
__global__ void __launch_bounds__(256, CO <= 16 ? 3 : 2) conv_adj_qbar_rb_kernel(const float* __restrict__ Pbar, ConvStep cs, int M,
                                                               const float* __restrict__ gseed,
                                                               const float* __restrict__ b, float* __restrict__ Qbar) {
    extern __shared__ float4 rb_w4[];
    float* wsh = reinterpret_cast<float*>(rb_w4);
    // wsh[((ky kw + kx) Ci + ci) CO + co] = W[co, ci, ky, kx]
    const int taps = cs.kh * cs.kw;
    const int nwt = taps * cs.Ci * CO;
    for (int i = threadIdx.x; i < nwt; i += blockDim.x) {
        const int co = i % CO, rest = i / CO;
        const int ci = rest % cs.Ci, tap = rest / cs.Ci;
        wsh[i] = cs.Wc[((size_t)co * taps + tap) * cs.Ci + ci];
    }
    __syncthreads();
    const int nq = cs.in_h * cs.in_w;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < (int64_t)M * nq;
         idx += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(idx / nq), q = (int)(idx - (int64_t)r * nq);
    const int qy = q / cs.in_w, qx = q - (q / cs.in_w) * cs.in_w;
    const float* prow = Pbar + (size_t)r * cs.out_h * cs.out_w * cs.Ci;
    float acc[CO];
#pragma unroll
    for (int c = 0; c < CO; ++c) acc[c] = 0.f;
    for (int ky = 0; ky < cs.kh; ++ky) {
        const int vy = qy * cs.sh + ky - cs.cy;
        if (vy < 0 || vy >= cs.out_h) continue;
        for (int kx = 0; kx < cs.kw; ++kx) {
            const int vx = qx * cs.sw + kx - cs.cx;
            if (vx < 0 || vx >= cs.out_w) continue;
            const float4* p4 = reinterpret_cast<const float4*>(prow + ((size_t)vy * cs.out_w + vx) * cs.Ci);
            const float* w = wsh + (size_t)(ky * cs.kw + kx) * cs.Ci * CO;
            for (int c4 = 0; c4 < cs.Ci / 4; ++c4) {
                const float4 pv = __ldg(p4 + c4);
                const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float4* wr = reinterpret_cast<const float4*>(w + (size_t)(c4 * 4 + t) * CO);
#pragma unroll
                    for (int c = 0; c < CO / 4; ++c) {
                        const float4 wv = wr[c];
                        acc[4 * c + 0] = fmaf(pa[t], wv.x, acc[4 * c + 0]);
                        acc[4 * c + 1] = fmaf(pa[t], wv.y, acc[4 * c + 1]);
                        acc[4 * c + 2] = fmaf(pa[t], wv.z, acc[4 * c + 2]);
                        acc[4 * c + 3] = fmaf(pa[t], wv.w, acc[4 * c + 3]);
                    }
                }
            }
        }
    }
    const float g = gseed[r];
    float* out = Qbar + (size_t)idx * CO;
#pragma unroll
    for (int c = 0; c < CO; c += 4)
        *reinterpret_cast<float4*>(out + c) = make_float4(acc[c] + g * b[c], acc[c + 1] + g * b[c + 1],
                                                          acc[c + 2] + g * b[c + 2], acc[c + 3] + g * b[c + 3]);
    }
}

void launch_conv_adj_qbar_rb(const float* Pbar, const ConvStep& cs, int M, const float* gseed, const float* b,
                             float* Qbar, cudaStream_t s) {
    const int64_t total = (int64_t)M * cs.in_h * cs.in_w;
    if (total == 0) return;
    if (!conv_adj_rb_ok(cs)) throw std::invalid_argument("conv_adj_qbar_rb: unsupported step");
    const size_t smem = (size_t)cs.kh * cs.kw * cs.Co * cs.Ci * 4;
    // Persistent blocks: the weights are staged once per block.
    const int64_t items = ceil_div(total, 256);
    if (cs.Co == 8)
        conv_adj_qbar_rb_kernel<8><<<rb_grid(conv_adj_qbar_rb_kernel<8>, smem, items), 256, smem, s>>>(
            Pbar, cs, M, gseed, b, Qbar);
    else if (cs.Co == 16)
        conv_adj_qbar_rb_kernel<16><<<rb_grid(conv_adj_qbar_rb_kernel<16>, smem, items), 256, smem, s>>>(
            Pbar, cs, M, gseed, b, Qbar);
    else
        conv_adj_qbar_rb_kernel<32><<<rb_grid(conv_adj_qbar_rb_kernel<32>, smem, items), 256, smem, s>>>(
            Pbar, cs, M, gseed, b, Qbar);
    LB_LAUNCH();
}

int relax_window_chunks(const WinGeo& g) { return ceil_div(g.size(), 1024); }

// 256 threads x 4 consecutive elements (one pixel's channels when C % 4 == 0).
__global__ void __launch_bounds__(256) relax_window_kernel(float* __restrict__ P, ConvRelaxEpi e, int M,
                                                           int nchunk, float* __restrict__ partial) {
    __shared__ float sh[8];
    const int r = (int)(blockIdx.x / nchunk), chunk = (int)(blockIdx.x % nchunk);
    const int nw = e.g.size();
    const int j0 = chunk * 1024 + threadIdx.x * 4;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    int oy, ox;
    win_origin(e.g, e.rows.row_id[rr], oy, ox);
    float part = 0.f;
    if (j0 < nw) {
        const size_t at = (size_t)r * nw + j0;
        float4 p4 = *reinterpret_cast<const float4*>(P + at);
        if (e.addend) {
            const float4 a = *reinterpret_cast<const float4*>(e.addend + at);
            p4 = make_float4(p4.x + a.x, p4.y + a.y, p4.z + a.z, p4.w + a.w);
            *reinterpret_cast<float4*>(P + at) = p4;
        }
        const float Pv[4] = {p4.x, p4.y, p4.z, p4.w};
        const int nu0 = win_neuron(e.g, oy, ox, j0);  // the 4 elements share a pixel
        float Qv[4] = {0.f, 0.f, 0.f, 0.f};
        if (nu0 >= 0) {
            const size_t bj = (size_t)bx * e.rp.n + nu0;
            const float4 s4 = *reinterpret_cast<const float4*>(e.rp.slope_lo + bj);
            const float4 k4 = *reinterpret_cast<const float4*>(e.rp.k_up + bj);
            const float4 b4 = *reinterpret_cast<const float4*>(e.rp.b_up + bj);
            const uchar4 f4 = *reinterpret_cast<const uchar4*>(e.rp.flags + bj);
            float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e.alpha && ((f4.x | f4.y | f4.z | f4.w) & RF_USE_ALPHA))
                a4 = *reinterpret_cast<const float4*>(e.alpha + at);
            const float Av[4] = {a4.x, a4.y, a4.z, a4.w};
            const float sl[4] = {s4.x, s4.y, s4.z, s4.w}, ku[4] = {k4.x, k4.y, k4.z, k4.w},
                        bu[4] = {b4.x, b4.y, b4.z, b4.w};
            const uint8_t fl[4] = {f4.x, f4.y, f4.z, f4.w};
            const int c0 = j0 % e.g.C;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float sv = (e.alpha && (fl[i] & RF_USE_ALPHA)) ? Av[i] : sl[i];
                Qv[i] = relax_q(Pv[i], p, sv, ku[i], bu[i], part);
                if (e.b_next) part = fmaf(Qv[i], e.b_next[c0 + i], part);
            }
        }
        *reinterpret_cast<float4*>(e.Q + at) = make_float4(Qv[0], Qv[1], Qv[2], Qv[3]);
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) partial[(size_t)chunk * M + r] = tot;
}

void launch_relax_window(float* P, const ConvRelaxEpi& e, int M, float* partial, cudaStream_t s) {
    if (M == 0) return;
    if (e.g.C % 4 != 0) throw std::invalid_argument("relax_window: channels must be a multiple of 4");
    const int nchunk = relax_window_chunks(e.g);
    relax_window_kernel<<<(unsigned)((int64_t)M * nchunk), 256, 0, s>>>(P, e, M, nchunk, partial);
    LB_LAUNCH();
}

// ============================================================== adjoint
__global__ void win_input_seed_kernel(RowMap rows, int M, WinGeo g, int form, const uint8_t* __restrict__ sign,
                                      const float* __restrict__ gseed, const float* __restrict__ xl,
                                      const float* __restrict__ xu, float* __restrict__ out) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nw = g.size();
    if (idx >= (int64_t)M * nw) return;
    const int r = (int)(idx / nw), j = (int)(idx - (int64_t)r * nw);
    int p, rr;
    row_split(r, rows.R, p, rr);
    const int bx = rows.row_box[rr];
    int oy, ox;
    win_origin(g, rows.row_id[rr], oy, ox);
    const int nu = win_neuron(g, oy, ox, j);
    float v = 0.f;
    if (nu >= 0) {
        const int n0 = g.C * g.H * g.W;
        const float l = xl[(size_t)bx * n0 + nu], u = xu[(size_t)bx * n0 + nu];
        const uint8_t sg = sign[idx];
        const float gr = gseed[r];
        if (form == CONC_PATCHES) {
            const float c = (u + l) / 2.0f, d = (u - l) / 2.0f;
            const float sgn = (sg & 1) ? 1.f : ((sg & 2) ? -1.f : 0.f);
            v = p == 0 ? gr * c - gr * d * sgn : gr * c + gr * d * sgn;
        } else {
            const float xa = p == 0 ? l : u, xb = p == 0 ? u : l;
            v = ((sg & 1) ? gr * xa : 0.f) + ((sg & 2) ? gr * xb : 0.f);
        }
    }
    out[idx] = v;
}

void launch_win_input_seed(const RowMap& rows, int M, const WinGeo& g, int form, const uint8_t* sign,
                           const float* gseed, const float* xl, const float* xu, float* Pbar0,
                           cudaStream_t s) {
    const int64_t total = (int64_t)M * g.size();
    if (total == 0) return;
    win_input_seed_kernel<<<ceil_div(total, 256), 256, 0, s>>>(rows, M, g, form, sign, gseed, xl, xu, Pbar0);
    LB_LAUNCH();
}

__global__ void conv_adj_qbar_kernel(const float* __restrict__ Pbar, ConvStep cs, int M,
                                     const float* __restrict__ gseed, const float* __restrict__ b,
                                     float* __restrict__ Qbar) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nin = cs.in_h * cs.in_w * cs.Co;
    if (idx >= (int64_t)M * nin) return;
    const int r = (int)(idx / nin), j = (int)(idx - (int64_t)r * nin);
    const int co = j % cs.Co, pix = j / cs.Co;
    const int qy = pix / cs.in_w, qx = pix - qy * cs.in_w;
    const float* prow = Pbar + (size_t)r * cs.out_h * cs.out_w * cs.Ci;
    float acc = 0.f;
    for (int ky = 0; ky < cs.kh; ++ky) {
        const int vy = qy * cs.sh + ky - cs.cy;
        if (vy < 0 || vy >= cs.out_h) continue;
        for (int kx = 0; kx < cs.kw; ++kx) {
            const int vx = qx * cs.sw + kx - cs.cx;
            if (vx < 0 || vx >= cs.out_w) continue;
            const float* pb = prow + ((size_t)vy * cs.out_w + vx) * cs.Ci;
            const float* w = cs.Wc + ((size_t)(co * cs.kh + ky) * cs.kw + kx) * cs.Ci;
            for (int ci = 0; ci < cs.Ci; ++ci) acc = fmaf(pb[ci], w[ci], acc);
        }
    }
    Qbar[idx] = acc + gseed[r] * b[co];
}

void launch_conv_adj_qbar(const float* Pbar, const ConvStep& cs, int M, const float* gseed, const float* b,
                          float* Qbar, cudaStream_t s) {
    const int64_t total = (int64_t)M * cs.in_h * cs.in_w * cs.Co;
    if (total == 0) return;
    conv_adj_qbar_kernel<<<ceil_div(total, 256), 256, 0, s>>>(Pbar, cs, M, gseed, b, Qbar);
    LB_LAUNCH();
}

// Persistent blocks walk the rows; each block first tabulates, per window
// pixel, its (wy, wx) and its pixel offset in the phase-split Pbar layout,
// so the per-element work has no integer division.
constexpr int WIN_MAX_PIX = 2048;

__global__ void __launch_bounds__(256) relax_adjoint_win_kernel(EpiRelaxAdj e, WinGeo g,
                                                                const float* __restrict__ Qbar, int M) {
    __shared__ short2 pxy[WIN_MAX_PIX];
    __shared__ int pdo[WIN_MAX_PIX];
    const int npix = g.wh * g.ww, nw = g.size(), C = g.C;
    for (int q = threadIdx.x; q < npix; q += blockDim.x) {
        const int wy = q / g.ww, wx = q - (q / g.ww) * g.ww;
        pxy[q] = make_short2((short)wy, (short)wx);
        if (e.ps.s) {
            const int vy = wy + e.ps.cy, vx = wx + e.ps.cx;
            const int plane = (vy % e.ps.s) * e.ps.s + vx % e.ps.s;
            pdo[q] = ((plane * e.ps.nty + vy / e.ps.s - e.ps.tlo_y) * e.ps.ntx + vx / e.ps.s - e.ps.tlo_x) * C;
        } else {
            pdo[q] = q * C;
        }
    }
    __syncthreads();
    const bool cpow2 = (C & (C - 1)) == 0;
    const int cshift = __ffs(C) - 1;
    for (int r = blockIdx.x; r < M; r += gridDim.x) {
        int p, rr;
        row_split(r, e.rows.R, p, rr);
        const int bx = e.rows.row_box[rr];
        int oy, ox;
        win_origin(g, e.rows.row_id[rr], oy, ox);
        const float gr = e.gseed[r];
        const bool act = e.active && e.active[bx];
        const int64_t prow = e.ps.s ? (int64_t)r * e.ps.row_stride : (int64_t)r * nw;
        if ((C & 3) == 0) {
            // Four channels of one pixel per thread: float4 traffic.
            for (int j = threadIdx.x * 4; j < nw; j += blockDim.x * 4) {
                const int c = cpow2 ? (j & (C - 1)) : j % C, q = cpow2 ? (j >> cshift) : j / C;
                const short2 w2 = pxy[q];
                const int y = oy + w2.x, x = ox + w2.y;
                const int64_t idx = (int64_t)r * nw + j;
                float* pd = e.Pbar ? e.Pbar + prow + pdo[q] + c : nullptr;
                if ((unsigned)y >= (unsigned)g.H || (unsigned)x >= (unsigned)g.W) {
                    if (pd) *reinterpret_cast<float4*>(pd) = make_float4(0.f, 0.f, 0.f, 0.f);
                    continue;
                }
                const size_t bj = (size_t)bx * e.rp.n + (y * g.W + x) * C + c;
                const float4 q4 = *reinterpret_cast<const float4*>(Qbar + idx);
                const float4 p4 = *reinterpret_cast<const float4*>(e.P_saved + idx);
                const float4 s4 = *reinterpret_cast<const float4*>(e.rp.slope_lo + bj);
                const float4 k4 = *reinterpret_cast<const float4*>(e.rp.k_up + bj);
                const float4 b4 = *reinterpret_cast<const float4*>(e.rp.b_up + bj);
                const uchar4 f4 = *reinterpret_cast<const uchar4*>(e.rp.flags + bj);
                const uint8_t fl[4] = {f4.x, f4.y, f4.z, f4.w};
                const uint8_t fany = f4.x | f4.y | f4.z | f4.w;
                const bool adam = e.adam_m && act && (fany & RF_ASET);
                float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (e.alpha && (adam || (fany & RF_USE_ALPHA))) a4 = *reinterpret_cast<const float4*>(e.alpha + idx);
                float4 m4 = make_float4(0.f, 0.f, 0.f, 0.f), v4 = m4;
                if (adam) {
                    m4 = *reinterpret_cast<const float4*>(e.adam_m + idx);
                    v4 = *reinterpret_cast<const float4*>(e.adam_v + idx);
                }
                const float Qv[4] = {q4.x, q4.y, q4.z, q4.w}, Pv[4] = {p4.x, p4.y, p4.z, p4.w};
                const float sl[4] = {s4.x, s4.y, s4.z, s4.w}, ku[4] = {k4.x, k4.y, k4.z, k4.w},
                            bu[4] = {b4.x, b4.y, b4.z, b4.w};
                float Av[4] = {a4.x, a4.y, a4.z, a4.w}, Mv[4] = {m4.x, m4.y, m4.z, m4.w},
                      Vv[4] = {v4.x, v4.y, v4.z, v4.w}, out[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const bool use_alpha = (fl[i] & RF_USE_ALPHA) != 0, un = (fl[i] & RF_UNSTABLE) != 0;
                    const float sv = (e.alpha && use_alpha) ? Av[i] : sl[i];
                    const bool pos = Pv[i] >= 0.f, neg = Pv[i] <= 0.f;
                    const float sP = p == 0 ? sv : ku[i], sN = p == 0 ? ku[i] : sv;
                    const float bP = p == 0 ? 0.f : bu[i], bN = p == 0 ? bu[i] : 0.f;
                    const float dq = (pos ? sP : 0.f) + (neg ? sN : 0.f);
                    const float db = (pos ? bP : 0.f) + (neg ? bN : 0.f);
                    out[i] = Qv[i] * dq + gr * db;
                    const float Pp = fmaxf(Pv[i], 0.f), Pn = fminf(Pv[i], 0.f);
                    if (un) {
                        const float kv = Qv[i] * (p == 0 ? Pn : Pp), bv = gr * (p == 0 ? Pn : Pp);
                        if (kv != 0.f) atomicAdd(e.kbar_d + bj + i, (double)kv);
                        if (bv != 0.f) atomicAdd(e.bbar_d + bj + i, (double)bv);
                    }
                    if (adam) {
                        const float ag = use_alpha ? Qv[i] * (p == 0 ? Pp : Pn) : 0.f;
                        Av[i] = adam_clip_update(Av[i], ag, Mv[i], Vv[i], e.adam_step, e.adam_bc2_sqrt);
                    }
                }
                if (pd) *reinterpret_cast<float4*>(pd) = make_float4(out[0], out[1], out[2], out[3]);
                if (adam) {
                    *reinterpret_cast<float4*>(e.alpha + idx) = make_float4(Av[0], Av[1], Av[2], Av[3]);
                    *reinterpret_cast<float4*>(e.adam_m + idx) = make_float4(Mv[0], Mv[1], Mv[2], Mv[3]);
                    *reinterpret_cast<float4*>(e.adam_v + idx) = make_float4(Vv[0], Vv[1], Vv[2], Vv[3]);
                }
            }
            continue;
        }
        for (int j = threadIdx.x; j < nw; j += blockDim.x) {
            const int c = cpow2 ? (j & (C - 1)) : j % C, q = cpow2 ? (j >> cshift) : j / C;
            const short2 w2 = pxy[q];
            const int y = oy + w2.x, x = ox + w2.y;
            const int64_t idx = (int64_t)r * nw + j;
            const int64_t pdst = prow + pdo[q] + c;
            if ((unsigned)y >= (unsigned)g.H || (unsigned)x >= (unsigned)g.W) {
                if (e.Pbar) e.Pbar[pdst] = 0.f;
                continue;
            }
            const size_t bj = (size_t)bx * e.rp.n + (y * g.W + x) * C + c;
            const uint8_t f = e.rp.flags[bj];
            const float sl = e.rp.slope_lo[bj], k = e.rp.k_up[bj], b = e.rp.b_up[bj];
            const bool use_alpha = (f & RF_USE_ALPHA) != 0, un = (f & RF_UNSTABLE) != 0;
            const float Qb = Qbar[idx];
            const float P = e.P_saved[idx];
            const bool adam = e.adam_m && act && (f & RF_ASET);
            const float a = (e.alpha && (use_alpha || adam)) ? e.alpha[idx] : 0.f;
            const float sv = (e.alpha && use_alpha) ? a : sl;
            const bool pos = P >= 0.f, neg = P <= 0.f;
            const float sP = p == 0 ? sv : k, sN = p == 0 ? k : sv;
            const float bP = p == 0 ? 0.f : b, bN = p == 0 ? b : 0.f;
            if (e.Pbar) {
                const float dq = (pos ? sP : 0.f) + (neg ? sN : 0.f);
                const float db = (pos ? bP : 0.f) + (neg ? bN : 0.f);
                e.Pbar[pdst] = Qb * dq + gr * db;
            }
            const float Pp = fmaxf(P, 0.f), Pn = fminf(P, 0.f);
            if (un) {
                const float kv = Qb * (p == 0 ? Pn : Pp), bv = gr * (p == 0 ? Pn : Pp);
                if (kv != 0.f) atomicAdd(e.kbar_d + bj, (double)kv);
                if (bv != 0.f) atomicAdd(e.bbar_d + bj, (double)bv);
            }
            if (adam) {
                const float ag = use_alpha ? Qb * (p == 0 ? Pp : Pn) : 0.f;
                float mm = e.adam_m[idx], vv = e.adam_v[idx];
                e.alpha[idx] = adam_clip_update(a, ag, mm, vv, e.adam_step, e.adam_bc2_sqrt);
                e.adam_m[idx] = mm;
                e.adam_v[idx] = vv;
            }
        }
    }
}

void launch_relax_adjoint_win(const EpiRelaxAdj& e, const WinGeo& g, const float* Qbar, int M, cudaStream_t s) {
    if ((int64_t)M * g.size() == 0) return;
    if (g.wh * g.ww > WIN_MAX_PIX) throw std::invalid_argument("relax_adjoint_win: window too large");
    int dev = 0, sms = 0;
    LB_CUDA(cudaGetDevice(&dev));
    LB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = std::min(M, sms * 8);
    relax_adjoint_win_kernel<<<grid, 256, 0, s>>>(e, g, Qbar, M);
    LB_LAUNCH();
}

// ============================================================== first conv layer
namespace {
constexpr int FK = 3, FC = 3;  // kernel 3x3 over 3 input channels, stride 1
}  // namespace

// Shared seed window of the first-conv adjoint: a zero halo of FK rows /
// columns on each side, plus a segment of slack columns on the right so that
// the last row segment's reads stay inside.
constexpr int FSEG = 16;
__host__ __device__ inline int first_seed_pw(int out_w) { return out_w + 2 * FK + FSEG; }
__host__ __device__ inline int first_seed_ph(int out_h) { return out_h + 2 * FK + 1; }

bool first_conv_fast(const ConvStep& cs) {
    return cs.kh == FK && cs.kw == FK && cs.Ci == FC && cs.Co <= 32 && cs.sh == 1 && cs.sw == 1 && cs.cy <= FK &&
           cs.cx <= FK && first_seed_ph(cs.out_h) * first_seed_pw(cs.out_w) * FC * 4 <= 48 * 1024;
}

// Warp task: one output row segment of FSEG pixels.  Lane = conv output
// channel co (its 27 weights in registers); every loaded data column is used
// by the three x-taps of its neighbouring pixels.  The per-lane partial sums
// (FSEG pixels x 3 channels) are reduced across lanes by a transposed
// butterfly: after the rounds over lane bits 16, 8, 4, 2 lane L holds the
// three channels of pixel L >> 1, completed by a final exchange with L ^ 1.

__global__ void __launch_bounds__(256) first_convT_conc_kernel(const float* __restrict__ A, ConvStep cs, int M,
                                                               ConvConcEpi e, float* __restrict__ partial) {
    __shared__ float sh[8];
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    int oy, ox;
    win_origin(e.g, e.rows.row_id[rr], oy, ox);
    const int n0 = e.g.C * e.g.H * e.g.W;
    const int nin = cs.in_h * cs.in_w * cs.Co;
    const int nw = e.g.size();
    const float* Arow = A + (size_t)r * nin;
    const int co = lane;  // Co <= 32
    const bool cok = co < cs.Co;
    float w[FK * FK * FC];
#pragma unroll
    for (int t = 0; t < FK * FK; ++t)
#pragma unroll
        for (int ci = 0; ci < FC; ++ci) w[t * FC + ci] = cok ? cs.Wk[((size_t)t * cs.Co + co) * FC + ci] : 0.f;
    float part = 0.f;
    const int nseg = (cs.out_w + FSEG - 1) / FSEG;
    for (int task = warp; task < cs.out_h * nseg; task += 8) {
        const int vy = task / nseg, x0 = (task - (task / nseg) * nseg) * FSEG;
        float acc[FSEG * FC];
#pragma unroll
        for (int i = 0; i < FSEG * FC; ++i) acc[i] = 0.f;
#pragma unroll
        for (int c = 0; c < FSEG + FK - 1; ++c) {
            const int qx = x0 + cs.cx - (FK - 1) + c;
            const bool xok = cok && qx >= 0 && qx < cs.in_w;
            float a[FK];
#pragma unroll
            for (int ky = 0; ky < FK; ++ky) {
                const int qy = vy + cs.cy - ky;
                a[ky] = (xok && qy >= 0 && qy < cs.in_h) ? Arow[((size_t)qy * cs.in_w + qx) * cs.Co + co] : 0.f;
            }
#pragma unroll
            for (int kx = 0; kx < FK; ++kx) {
                const int pl = c - (FK - 1) + kx;
                if (pl < 0 || pl >= FSEG) continue;
#pragma unroll
                for (int ky = 0; ky < FK; ++ky)
#pragma unroll
                    for (int ci = 0; ci < FC; ++ci)
                        acc[pl * FC + ci] = fmaf(a[ky], w[(ky * FK + kx) * FC + ci], acc[pl * FC + ci]);
            }
        }
        // Transposed butterfly over lane bits 16, 8, 4, 2.
        float v24[24], v12[12], v6[6], v3[3];
        {
            const bool hi = lane & 16;
#pragma unroll
            for (int i = 0; i < 24; ++i) {
                const float keep = hi ? acc[24 + i] : acc[i], send = hi ? acc[i] : acc[24 + i];
                v24[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
            }
        }
        {
            const bool hi = lane & 8;
#pragma unroll
            for (int i = 0; i < 12; ++i) {
                const float keep = hi ? v24[12 + i] : v24[i], send = hi ? v24[i] : v24[12 + i];
                v12[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
        }
        {
            const bool hi = lane & 4;
#pragma unroll
            for (int i = 0; i < 6; ++i) {
                const float keep = hi ? v12[6 + i] : v12[i], send = hi ? v12[i] : v12[6 + i];
                v6[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
        }
        {
            const bool hi = lane & 2;
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                const float keep = hi ? v6[3 + i] : v6[i], send = hi ? v6[i] : v6[3 + i];
                v3[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
            }
        }
#pragma unroll
        for (int i = 0; i < 3; ++i) v3[i] += __shfl_xor_sync(0xffffffffu, v3[i], 1);
        const int vx = x0 + (lane >> 1);
        if ((lane & 1) == 0 && vx < cs.out_w) {
#pragma unroll
            for (int ci = 0; ci < FC; ++ci) {
                const float P = v3[ci];
                const int j = (vy * cs.out_w + vx) * FC + ci;
                const int nu = win_neuron(e.g, oy, ox, j);
                uint8_t sg = 0;
                if (nu >= 0) {
                    const float xl = e.xl[(size_t)bx * n0 + nu], xu = e.xu[(size_t)bx * n0 + nu];
                    if (e.form == CONC_PATCHES) {
                        const float c = (xu + xl) / 2.0f, d = (xu - xl) / 2.0f;
                        part += p == 0 ? fmaf(P, c, -fabsf(P) * d) : fmaf(P, c, fabsf(P) * d);
                        sg = (uint8_t)((P > 0.f ? 1 : 0) | (P < 0.f ? 2 : 0));
                    } else {
                        const float xa = p == 0 ? xl : xu, xb = p == 0 ? xu : xl;
                        part += fmaxf(P, 0.f) * xa + fminf(P, 0.f) * xb;
                        sg = (uint8_t)((P >= 0.f ? 1 : 0) | (P <= 0.f ? 2 : 0));
                    }
                }
                if (e.sign) e.sign[(size_t)r * nw + j] = sg;
            }
        }
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) partial[r] = tot;
}

void launch_first_convT_conc(const float* A, const ConvStep& cs, int M, const ConvConcEpi& e, float* partial,
                             cudaStream_t s) {
    if (M == 0) return;
    if (cs.Co > 32) throw std::invalid_argument("first_convT_conc: Co > 32");
    first_convT_conc_kernel<<<M, 256, 0, s>>>(A, cs, M, e, partial);
    LB_LAUNCH();
}

__global__ void __launch_bounds__(256) first_conv_adj_kernel(RowMap rows, int M, WinGeo g0, int form,
                                                             const uint8_t* __restrict__ sign,
                                                             const float* __restrict__ gseed,
                                                             const float* __restrict__ xl,
                                                             const float* __restrict__ xu, ConvStep cs,
                                                             const float* __restrict__ b,
                                                             float* __restrict__ Qbar) {
    extern __shared__ float sP[];  // seed window (first_seed_ph x first_seed_pw x FC)
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int PW = first_seed_pw(cs.out_w), PH = first_seed_ph(cs.out_h);
    for (int i = threadIdx.x; i < PH * PW * FC; i += blockDim.x) sP[i] = 0.f;
    __syncthreads();
    int p, rr;
    row_split(r, rows.R, p, rr);
    const int bx = rows.row_box[rr];
    int oy, ox;
    win_origin(g0, rows.row_id[rr], oy, ox);
    const int n0 = g0.C * g0.H * g0.W;
    const int nw = g0.size();
    const float gr = gseed[r];
    for (int j = threadIdx.x; j < nw; j += blockDim.x) {
        const int nu = win_neuron(g0, oy, ox, j);
        float v = 0.f;
        if (nu >= 0) {
            const float l = xl[(size_t)bx * n0 + nu], u = xu[(size_t)bx * n0 + nu];
            const uint8_t sg = sign[(size_t)r * nw + j];
            if (form == CONC_PATCHES) {
                const float c = (u + l) / 2.0f, d = (u - l) / 2.0f;
                const float sgn = (sg & 1) ? 1.f : ((sg & 2) ? -1.f : 0.f);
                v = p == 0 ? gr * c - gr * d * sgn : gr * c + gr * d * sgn;
            } else {
                const float xa = p == 0 ? l : u, xbv = p == 0 ? u : l;
                v = ((sg & 1) ? gr * xa : 0.f) + ((sg & 2) ? gr * xbv : 0.f);
            }
        }
        const int ci = j % FC, pix = j / FC;
        const int vy = pix / cs.out_w, vx = pix - (pix / cs.out_w) * cs.out_w;
        sP[((vy + FK) * PW + vx + FK) * FC + ci] = v;
    }
    __syncthreads();
    // Warp task: FSEG consecutive output pixels of one row; lane = co.  Each
    // seed column is read once and used by the three x-taps that touch it.
    const int co = lane;  // Co <= 32
    const bool cok = co < cs.Co;
    float w[FK * FK * FC];
#pragma unroll
    for (int t = 0; t < FK * FK * FC; ++t) w[t] = cok ? cs.Wc[(size_t)co * FK * FK * FC + t] : 0.f;
    const float gb = cok ? gr * b[co] : 0.f;
    const int nseg = (cs.in_w + FSEG - 1) / FSEG;
    for (int task = warp; task < cs.in_h * nseg; task += 8) {
        const int qy = task / nseg, x0 = (task - (task / nseg) * nseg) * FSEG;
        const float* base = sP + ((qy - cs.cy + FK) * PW + x0 - cs.cx + FK) * FC;
        float acc[FSEG];
#pragma unroll
        for (int i = 0; i < FSEG; ++i) acc[i] = 0.f;
#pragma unroll
        for (int c = 0; c < FSEG + FK - 1; ++c) {
            float pv[FK * FC];
#pragma unroll
            for (int ky = 0; ky < FK; ++ky)
#pragma unroll
                for (int ci = 0; ci < FC; ++ci) pv[ky * FC + ci] = base[(ky * PW + c) * FC + ci];
#pragma unroll
            for (int kx = 0; kx < FK; ++kx) {
                const int ql = c - kx;
                if (ql < 0 || ql >= FSEG) continue;
#pragma unroll
                for (int ky = 0; ky < FK; ++ky)
#pragma unroll
                    for (int ci = 0; ci < FC; ++ci)
                        acc[ql] = fmaf(pv[ky * FC + ci], w[(ky * FK + kx) * FC + ci], acc[ql]);
            }
        }
        if (cok) {
#pragma unroll
            for (int i = 0; i < FSEG; ++i)
                if (x0 + i < cs.in_w) Qbar[((size_t)r * cs.in_h * cs.in_w + qy * cs.in_w + x0 + i) * cs.Co + co] = acc[i] + gb;
        }
    }
}

void launch_first_conv_adj(const RowMap& rows, int M, const WinGeo& g0, int form, const uint8_t* sign,
                           const float* gseed, const float* xl, const float* xu, const ConvStep& cs,
                           const float* b, float* Qbar, cudaStream_t s) {
    if (M == 0) return;
    const size_t smem = (size_t)first_seed_ph(cs.out_h) * first_seed_pw(cs.out_w) * FC * 4;
    first_conv_adj_kernel<<<M, 256, smem, s>>>(rows, M, g0, form, sign, gseed, xl, xu, cs, b, Qbar);
    LB_LAUNCH();
}

// ============================================================== transposed-conv layers
__global__ void ibp_convt_kernel(ConvTStep ct, const float* __restrict__ bias, const float* __restrict__ in_l,
                                 const float* __restrict__ in_u, float* __restrict__ out_l,
                                 float* __restrict__ out_u, int B, bool relu_in) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nout = (int64_t)ct.Ho * ct.Wo * ct.Co;
    if (idx >= (int64_t)B * nout) return;
    const int bx = (int)(idx / nout);
    const int j = (int)(idx - (int64_t)bx * nout);
    const int co = j % ct.Co, pix = j / ct.Co;
    const int vy = pix / ct.Wo, vx = pix - (pix / ct.Wo) * ct.Wo;
    float c = 0.f, d = 0.f;
    for (int ky = 0; ky < ct.kh; ++ky) {
        const int ty = vy + ct.ph - ky;
        if (ty < 0 || ty % ct.sh) continue;
        const int qy = ty / ct.sh;
        if (qy >= ct.Hi) continue;
        for (int kx = 0; kx < ct.kw; ++kx) {
            const int tx = vx + ct.pw - kx;
            if (tx < 0 || tx % ct.sw) continue;
            const int qx = tx / ct.sw;
            if (qx >= ct.Wi) continue;
            const size_t base = (((size_t)bx * ct.Hi + qy) * ct.Wi + qx) * ct.Ci;
            const float* w = ct.Wa + ((size_t)(ky * ct.kw + kx) * ct.Co + co) * ct.Ci;
            for (int ci = 0; ci < ct.Ci; ++ci) {
                float l = in_l[base + ci], u = in_u[base + ci];
                if (relu_in) {
                    l = fmaxf(l, 0.f);
                    u = fmaxf(u, 0.f);
                }
                const float mid = (u + l) / 2.0f, diff = (u - l) / 2.0f;
                c = fmaf(mid, w[ci], c);
                d = fmaf(diff, fabsf(w[ci]), d);
            }
        }
    }
    c += bias ? bias[co] : 0.f;
    out_l[idx] = c - d;
    out_u[idx] = c + d;
}

void launch_ibp_convt(const ConvTStep& ct, const float* b, const float* in_l, const float* in_u, float* out_l,
                      float* out_u, int B, bool relu_in, cudaStream_t s) {
    const int64_t total = (int64_t)B * ct.Ho * ct.Wo * ct.Co;
    if (total == 0) return;
    ibp_convt_kernel<<<ceil_div(total, 256), 256, 0, s>>>(ct, b, in_l, in_u, out_l, out_u, B, relu_in);
    LB_LAUNCH();
}

__global__ void __launch_bounds__(256) convt_back_relax_kernel(const float* __restrict__ A, ConvTStep ct, int M,
                                                               ConvRelaxEpi e, int nchunk,
                                                               float* __restrict__ partial) {
    __shared__ float sh[8];
    const int r = (int)(blockIdx.x / nchunk), chunk = (int)(blockIdx.x % nchunk);
    const int nin = ct.Ho * ct.Wo * ct.Co;  // the rows' A at the layer's output
    const int nw = ct.Hi * ct.Wi * ct.Ci;
    const int j = chunk * 256 + threadIdx.x;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    float part = 0.f;
    if (j < nw) {
        const int ci = j % ct.Ci, pix = j / ct.Ci;
        const int qy = pix / ct.Wi, qx = pix - (pix / ct.Wi) * ct.Wi;
        const float* Arow = A + (size_t)r * nin;
        float P = 0.f;
        for (int ky = 0; ky < ct.kh; ++ky) {
            const int vy = qy * ct.sh - ct.ph + ky;
            if (vy < 0 || vy >= ct.Ho) continue;
            for (int kx = 0; kx < ct.kw; ++kx) {
                const int vx = qx * ct.sw - ct.pw + kx;
                if (vx < 0 || vx >= ct.Wo) continue;
                const float* a = Arow + ((size_t)vy * ct.Wo + vx) * ct.Co;
                const float* w = ct.Wg + (((size_t)ci * ct.kh + ky) * ct.kw + kx) * ct.Co;
                for (int co = 0; co < ct.Co; ++co) P = fmaf(a[co], w[co], P);
            }
        }
        const size_t at = (size_t)r * nw + j;
        if (e.P_save) e.P_save[at] = P;
        const size_t bj = (size_t)bx * e.rp.n + j;
        const float sl = (e.alpha && (e.rp.flags[bj] & RF_USE_ALPHA)) ? e.alpha[at] : e.rp.slope_lo[bj];
        const float Q = relax_q(P, p, sl, e.rp.k_up[bj], e.rp.b_up[bj], part);
        if (e.b_next) part = fmaf(Q, e.b_next[ci], part);
        e.Q[at] = Q;
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) partial[(size_t)chunk * M + r] = tot;
}

void launch_convt_back_relax(const float* A, const ConvTStep& ct, int M, const ConvRelaxEpi& e, float* partial,
                             cudaStream_t s) {
    if (M == 0) return;
    if (!e.g.full) throw std::invalid_argument("convt_back_relax: rows through a transposed conv are whole maps");
    const int nchunk = conv_chunks(e.g);
    convt_back_relax_kernel<<<(unsigned)((int64_t)M * nchunk), 256, 0, s>>>(A, ct, M, e, nchunk, partial);
    LB_LAUNCH();
}

__global__ void __launch_bounds__(256) convt_start_step_kernel(ConvStartStep st, ConvTStep ct) {
    __shared__ float sh[8];
    const int r = blockIdx.x;
    int p, rr;
    row_split(r, st.rows.R, p, rr);
    const int bx = st.rows.row_box[rr];
    const int id = st.rows.row_id[rr];  // HWC index at the layer's output
    const int co0 = id % ct.Co, pix0 = id / ct.Co;
    const int vy0 = pix0 / ct.Wo, vx0 = pix0 - (pix0 / ct.Wo) * ct.Wo;
    const int nw = ct.Hi * ct.Wi * ct.Ci;
    float part = 0.f;
    for (int j = threadIdx.x; j < nw; j += blockDim.x) {
        const int ci = j % ct.Ci, pix = j / ct.Ci;
        const int qy = pix / ct.Wi, qx = pix - (pix / ct.Wi) * ct.Wi;
        const int ky = vy0 + ct.ph - qy * ct.sh, kx = vx0 + ct.pw - qx * ct.sw;
        const float P = (ky >= 0 && ky < ct.kh && kx >= 0 && kx < ct.kw)
                            ? ct.Wg[(((size_t)ci * ct.kh + ky) * ct.kw + kx) * ct.Co + co0]
                            : 0.f;
        const size_t at = (size_t)r * nw + j;
        if (st.P_save) st.P_save[at] = P;
        const size_t bj = (size_t)bx * st.rp.n + j;
        const float sl = (st.alpha && (st.rp.flags[bj] & RF_USE_ALPHA)) ? st.alpha[at] : st.rp.slope_lo[bj];
        const float Q = relax_q(P, p, sl, st.rp.k_up[bj], st.rp.b_up[bj], part);
        if (st.b_next) part = fmaf(Q, st.b_next[ci], part);
        st.Q[at] = Q;
    }
    const float tot = block_sum256(part, sh);
    if (threadIdx.x == 0) st.bias_acc[r] = tot;
}

void launch_convt_start_step(const ConvStartStep& st, const ConvTStep& ct, cudaStream_t s) {
    if (st.M == 0) return;
    convt_start_step_kernel<<<st.M, 256, 0, s>>>(st, ct);
    LB_LAUNCH();
}

__global__ void convt_adj_qbar_kernel(const float* __restrict__ Pbar, ConvTStep ct, int M, float* __restrict__ Qbar) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nq = (int64_t)ct.Ho * ct.Wo * ct.Co;
    if (idx >= (int64_t)M * nq) return;
    const int r = (int)(idx / nq);
    const int j = (int)(idx - (int64_t)r * nq);
    const int co = j % ct.Co, pix = j / ct.Co;
    const int vy = pix / ct.Wo, vx = pix - (pix / ct.Wo) * ct.Wo;
    const float* prow = Pbar + (size_t)r * ct.Hi * ct.Wi * ct.Ci;
    float acc = 0.f;
    for (int ky = 0; ky < ct.kh; ++ky) {
        const int ty = vy + ct.ph - ky;
        if (ty < 0 || ty % ct.sh) continue;
        const int qy = ty / ct.sh;
        if (qy >= ct.Hi) continue;
        for (int kx = 0; kx < ct.kw; ++kx) {
            const int tx = vx + ct.pw - kx;
            if (tx < 0 || tx % ct.sw) continue;
            const int qx = tx / ct.sw;
            if (qx >= ct.Wi) continue;
            const float* pb = prow + ((size_t)qy * ct.Wi + qx) * ct.Ci;
            const float* w = ct.Wa + ((size_t)(ky * ct.kw + kx) * ct.Co + co) * ct.Ci;
            for (int ci = 0; ci < ct.Ci; ++ci) acc = fmaf(pb[ci], w[ci], acc);
        }
    }
    Qbar[idx] = acc;
}

void launch_convt_adj_qbar(const float* Pbar, const ConvTStep& ct, int M, float* Qbar, cudaStream_t s) {
    const int64_t total = (int64_t)M * ct.Ho * ct.Wo * ct.Co;
    if (total == 0) return;
    convt_adj_qbar_kernel<<<ceil_div(total, 256), 256, 0, s>>>(Pbar, ct, M, Qbar);
    LB_LAUNCH();
}

// ---- register-blocked transposed-conv layer steps ---------------------------
constexpr int CT_BACK_CB = 16, CT_ADJ_CB = 8;

bool convt_rb_ok(const ConvTStep& ct) {
    return ct.Ci % CT_BACK_CB == 0 && ct.Co % 4 == 0 &&
           (int64_t)ct.kh * ct.kw * ct.Co * CT_BACK_CB <= RB_MAX_W_FLOATS;
}

int convt_rb_chunks(const ConvTStep& ct) { return ceil_div(ct.Hi * ct.Wi, 256) * (ct.Ci / CT_BACK_CB); }

__global__ void __launch_bounds__(256, 3) convt_back_relax_rb_kernel(const float* __restrict__ A, ConvTStep ct, int M,
                                                                     ConvRelaxEpi e, int npc,
                                                                     float* __restrict__ partial) {
    extern __shared__ float4 rb_w4[];
    float* wsh = reinterpret_cast<float*>(rb_w4);
    __shared__ float red[8];
    const int cg = blockIdx.y, c0 = cg * CT_BACK_CB;
    const int taps = ct.kh * ct.kw;
    // wsh[(tap Co + co) CB + cc] = W[c0 + cc, co, tap]
    const int nwt = taps * ct.Co * CT_BACK_CB;
    for (int i = threadIdx.x; i < nwt; i += blockDim.x) {
        const int cc = i % CT_BACK_CB, rest = i / CT_BACK_CB;
        const int co = rest % ct.Co, tap = rest / ct.Co;
        wsh[i] = ct.Wg[((size_t)(c0 + cc) * taps + tap) * ct.Co + co];
    }
    __syncthreads();
    const int r = (int)(blockIdx.x / npc), pc = (int)(blockIdx.x % npc);
    const int npix = ct.Hi * ct.Wi;
    const int pix = pc * 256 + threadIdx.x;
    const int nw = npix * ct.Ci, nin = ct.Ho * ct.Wo * ct.Co;
    int p, rr;
    row_split(r, e.rows.R, p, rr);
    const int bx = e.rows.row_box[rr];
    float part = 0.f;
    if (pix < npix) {
        float acc[CT_BACK_CB];
#pragma unroll
        for (int c = 0; c < CT_BACK_CB; ++c) acc[c] = 0.f;
        const int qy = pix / ct.Wi, qx = pix - (pix / ct.Wi) * ct.Wi;
        const float* Arow = A + (size_t)r * nin;
        for (int ky = 0; ky < ct.kh; ++ky) {
            const int vy = qy * ct.sh - ct.ph + ky;
            if (vy < 0 || vy >= ct.Ho) continue;
            for (int kx = 0; kx < ct.kw; ++kx) {
                const int vx = qx * ct.sw - ct.pw + kx;
                if (vx < 0 || vx >= ct.Wo) continue;
                const float4* a4 = reinterpret_cast<const float4*>(Arow + ((size_t)vy * ct.Wo + vx) * ct.Co);
                const float* w = wsh + (size_t)(ky * ct.kw + kx) * ct.Co * CT_BACK_CB;
                for (int c4 = 0; c4 < ct.Co / 4; ++c4) {
                    const float4 a = __ldg(a4 + c4);
                    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float4* wr = reinterpret_cast<const float4*>(w + (size_t)(c4 * 4 + t) * CT_BACK_CB);
#pragma unroll
                        for (int c = 0; c < CT_BACK_CB / 4; ++c) {
                            const float4 wv = wr[c];
                            acc[4 * c + 0] = fmaf(av[t], wv.x, acc[4 * c + 0]);
                            acc[4 * c + 1] = fmaf(av[t], wv.y, acc[4 * c + 1]);
                            acc[4 * c + 2] = fmaf(av[t], wv.z, acc[4 * c + 2]);
                            acc[4 * c + 3] = fmaf(av[t], wv.w, acc[4 * c + 3]);
                        }
                    }
                }
            }
        }
        const size_t at0 = (size_t)r * nw + (size_t)pix * ct.Ci + c0;
        const size_t bj0 = (size_t)bx * e.rp.n + (size_t)pix * ct.Ci + c0;
#pragma unroll
        for (int c = 0; c < CT_BACK_CB; c += 4) {
            const float Pv[4] = {acc[c], acc[c + 1], acc[c + 2], acc[c + 3]};
            if (e.P_save) *reinterpret_cast<float4*>(e.P_save + at0 + c) = make_float4(Pv[0], Pv[1], Pv[2], Pv[3]);
            const float4 s4 = *reinterpret_cast<const float4*>(e.rp.slope_lo + bj0 + c);
            const float4 k4 = *reinterpret_cast<const float4*>(e.rp.k_up + bj0 + c);
            const float4 b4 = *reinterpret_cast<const float4*>(e.rp.b_up + bj0 + c);
            const uchar4 f4 = *reinterpret_cast<const uchar4*>(e.rp.flags + bj0 + c);
            float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e.alpha && ((f4.x | f4.y | f4.z | f4.w) & RF_USE_ALPHA))
                a4 = *reinterpret_cast<const float4*>(e.alpha + at0 + c);
            const float Av[4] = {a4.x, a4.y, a4.z, a4.w};
            const float sl[4] = {s4.x, s4.y, s4.z, s4.w}, ku[4] = {k4.x, k4.y, k4.z, k4.w},
                        bu[4] = {b4.x, b4.y, b4.z, b4.w};
            const uint8_t fl[4] = {f4.x, f4.y, f4.z, f4.w};
            float Qv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float sv = (e.alpha && (fl[i] & RF_USE_ALPHA)) ? Av[i] : sl[i];
                Qv[i] = relax_q(Pv[i], p, sv, ku[i], bu[i], part);
                if (e.b_next) part = fmaf(Qv[i], e.b_next[c0 + c + i], part);
            }
            *reinterpret_cast<float4*>(e.Q + at0 + c) = make_float4(Qv[0], Qv[1], Qv[2], Qv[3]);
        }
    }
    const float tot = block_sum256(part, red);
    if (threadIdx.x == 0) partial[(size_t)(cg * npc + pc) * M + r] = tot;
}

void launch_convt_back_relax_rb(const float* A, const ConvTStep& ct, int M, const ConvRelaxEpi& e, float* partial,
                                cudaStream_t s) {
    if (M == 0) return;
    if (!e.g.full || !convt_rb_ok(ct)) throw std::invalid_argument("convt_back_relax_rb: unsupported step");
    const int npc = ceil_div(ct.Hi * ct.Wi, 256);
    const size_t smem = (size_t)ct.kh * ct.kw * ct.Co * CT_BACK_CB * 4;
    const dim3 grid((unsigned)((int64_t)M * npc), (unsigned)(ct.Ci / CT_BACK_CB));
    convt_back_relax_rb_kernel<<<grid, 256, smem, s>>>(A, ct, M, e, npc, partial);
    LB_LAUNCH();
}

bool convt_adj_rb_ok(const ConvTStep& ct) {
    return ct.Co % CT_ADJ_CB == 0 && ct.Ci % 4 == 0 &&
           (int64_t)ct.kh * ct.kw * ct.Ci * CT_ADJ_CB <= RB_MAX_W_FLOATS;
}

__global__ void __launch_bounds__(256, 3) convt_adj_qbar_rb_kernel(const float* __restrict__ Pbar, ConvTStep ct, int M,
                                                                   float* __restrict__ Qbar) {
    extern __shared__ float4 rb_w4[];
    float* wsh = reinterpret_cast<float*>(rb_w4);
    const int c0 = blockIdx.y * CT_ADJ_CB;
    const int taps = ct.kh * ct.kw;
    // wsh[(tap Ci + ci) CB + cc] = Wa[tap][c0 + cc][ci]
    const int nwt = taps * ct.Ci * CT_ADJ_CB;
    for (int i = threadIdx.x; i < nwt; i += blockDim.x) {
        const int cc = i % CT_ADJ_CB, rest = i / CT_ADJ_CB;
        const int ci = rest % ct.Ci, tap = rest / ct.Ci;
        wsh[i] = ct.Wa[((size_t)tap * ct.Co + c0 + cc) * ct.Ci + ci];
    }
    __syncthreads();
    const int npix = ct.Ho * ct.Wo;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)M * npix) return;
    const int r = (int)(idx / npix), pix = (int)(idx - (int64_t)r * npix);
    const int vy = pix / ct.Wo, vx = pix - (pix / ct.Wo) * ct.Wo;
    const float* prow = Pbar + (size_t)r * ct.Hi * ct.Wi * ct.Ci;
    float acc[CT_ADJ_CB];
#pragma unroll
    for (int c = 0; c < CT_ADJ_CB; ++c) acc[c] = 0.f;
    for (int ky = 0; ky < ct.kh; ++ky) {
        const int ty = vy + ct.ph - ky;
        if (ty < 0 || ty % ct.sh) continue;
        const int qy = ty / ct.sh;
        if (qy >= ct.Hi) continue;
        for (int kx = 0; kx < ct.kw; ++kx) {
            const int tx = vx + ct.pw - kx;
            if (tx < 0 || tx % ct.sw) continue;
            const int qx = tx / ct.sw;
            if (qx >= ct.Wi) continue;
            const float4* p4 = reinterpret_cast<const float4*>(prow + ((size_t)qy * ct.Wi + qx) * ct.Ci);
            const float* w = wsh + (size_t)(ky * ct.kw + kx) * ct.Ci * CT_ADJ_CB;
            for (int c4 = 0; c4 < ct.Ci / 4; ++c4) {
                const float4 pv = __ldg(p4 + c4);
                const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float4* wr = reinterpret_cast<const float4*>(w + (size_t)(c4 * 4 + t) * CT_ADJ_CB);
#pragma unroll
                    for (int c = 0; c < CT_ADJ_CB / 4; ++c) {
                        const float4 wv = wr[c];
                        acc[4 * c + 0] = fmaf(pa[t], wv.x, acc[4 * c + 0]);
                        acc[4 * c + 1] = fmaf(pa[t], wv.y, acc[4 * c + 1]);
                        acc[4 * c + 2] = fmaf(pa[t], wv.z, acc[4 * c + 2]);
                        acc[4 * c + 3] = fmaf(pa[t], wv.w, acc[4 * c + 3]);
                    }
                }
            }
        }
    }
    float* out = Qbar + ((size_t)r * npix + pix) * ct.Co + c0;
#pragma unroll
    for (int c = 0; c < CT_ADJ_CB; c += 4)
        *reinterpret_cast<float4*>(out + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
}

void launch_convt_adj_qbar_rb(const float* Pbar, const ConvTStep& ct, int M, float* Qbar, cudaStream_t s) {
    const int64_t total = (int64_t)M * ct.Ho * ct.Wo;
    if (total == 0) return;
    if (!convt_adj_rb_ok(ct)) throw std::invalid_argument("convt_adj_qbar_rb: unsupported step");
    const size_t smem = (size_t)ct.kh * ct.kw * ct.Ci * CT_ADJ_CB * 4;
    const dim3 grid((unsigned)ceil_div(total, 256), (unsigned)(ct.Co / CT_ADJ_CB));
    convt_adj_qbar_rb_kernel<<<grid, 256, smem, s>>>(Pbar, ct, M, Qbar);
    LB_LAUNCH();
}

// ============================================================== skip edges
__global__ void skip_back_kernel(SkipStep k, RowMap rows, int M, const float* __restrict__ Q,
                                 float* __restrict__ S) {
    const int nw = k.go.size();
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)M * nw) return;
    const int r = (int)(idx / nw), j = (int)(idx - (int64_t)r * nw);
    const int ci = j % k.Ci, pix = j / k.Ci;
    const int vy = pix / k.go.ww, vx = pix - (pix / k.go.ww) * k.go.ww;
    const int ty = vy + k.cy, tx = vx + k.cx;
    float acc = 0.f;
    if (Q) {
        const float* q = Q + (size_t)r * k.gi.size();
        if (!k.Wk) {
            if ((unsigned)ty < (unsigned)k.gi.wh && (unsigned)tx < (unsigned)k.gi.ww)
                acc = q[((size_t)ty * k.gi.ww + tx) * k.Co + ci];
        } else {
            for (int ky = 0; ky < k.kh; ++ky) {
                const int dy = ty - ky;
                if (dy < 0 || dy % k.sh != 0 || dy / k.sh >= k.gi.wh) continue;
                for (int kx = 0; kx < k.kw; ++kx) {
                    const int dx = tx - kx;
                    if (dx < 0 || dx % k.sw != 0 || dx / k.sw >= k.gi.ww) continue;
                    const float* a = q + ((size_t)(dy / k.sh) * k.gi.ww + dx / k.sw) * k.Co;
                    const float* w = k.Wk + ((size_t)(ky * k.kw + kx) * k.Co) * k.Ci + ci;
                    for (int co = 0; co < k.Co; ++co) acc = fmaf(a[co], w[(size_t)co * k.Ci], acc);
                }
            }
        }
    } else {
        // One-hot start row: its neuron sits at pixel q0, channel co0 of level i.
        const int id = rows.row_id[r >= rows.R ? r - rows.R : r];
        const int co0 = id % k.Co, q0 = k.gi.full ? id / k.Co : 0;
        const int q0y = q0 / k.gi.ww, q0x = q0 - (q0 / k.gi.ww) * k.gi.ww;
        if (!k.Wk) {
            acc = (ty == q0y && tx == q0x && ci == co0) ? 1.f : 0.f;
        } else {
            const int ky = ty - q0y * k.sh, kx = tx - q0x * k.sw;
            if ((unsigned)ky < (unsigned)k.kh && (unsigned)kx < (unsigned)k.kw)
                acc = k.Wk[((size_t)(ky * k.kw + kx) * k.Co + co0) * k.Ci + ci];
        }
    }
    S[idx] += acc;
}

void launch_skip_back(const SkipStep& k, const RowMap& rows, int M, const float* Q, float* S, cudaStream_t s) {
    const int64_t total = (int64_t)M * k.go.size();
    if (total == 0) return;
    skip_back_kernel<<<ceil_div(total, 256), 256, 0, s>>>(k, rows, M, Q, S);
    LB_LAUNCH();
}

__global__ void skip_adj_kernel(SkipStep k, int M, const float* __restrict__ Pbar, PhaseSplit ps,
                                float* __restrict__ Qbar) {
    const int ni = k.gi.size(), nw = k.go.size();
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)M * ni) return;
    const int r = (int)(idx / ni), j = (int)(idx - (int64_t)r * ni);
    const int co = j % k.Co, pix = j / k.Co;
    const int qy = pix / k.gi.ww, qx = pix - (pix / k.gi.ww) * k.gi.ww;
    auto pb = [&](int vy, int vx, int c) {
        const int e = (vy * k.go.ww + vx) * k.Ci + c;
        return ps.s ? Pbar[phase_dst(ps, r, e)] : Pbar[(size_t)r * nw + e];
    };
    float acc = 0.f;
    if (!k.Wc) {
        const int vy = qy - k.cy, vx = qx - k.cx;
        if ((unsigned)vy < (unsigned)k.go.wh && (unsigned)vx < (unsigned)k.go.ww) acc = pb(vy, vx, co);
    } else {
        for (int ky = 0; ky < k.kh; ++ky) {
            const int vy = qy * k.sh + ky - k.cy;
            if ((unsigned)vy >= (unsigned)k.go.wh) continue;
            for (int kx = 0; kx < k.kw; ++kx) {
                const int vx = qx * k.sw + kx - k.cx;
                if ((unsigned)vx >= (unsigned)k.go.ww) continue;
                const float* w = k.Wc + ((size_t)(co * k.kh + ky) * k.kw + kx) * k.Ci;
                for (int ci = 0; ci < k.Ci; ++ci) acc = fmaf(pb(vy, vx, ci), w[ci], acc);
            }
        }
    }
    Qbar[idx] += acc;
}

void launch_skip_adj(const SkipStep& k, const RowMap& rows, int M, const float* Pbar, const PhaseSplit& ps,
                     float* Qbar, cudaStream_t s) {
    (void)rows;
    const int64_t total = (int64_t)M * k.gi.size();
    if (total == 0) return;
    skip_adj_kernel<<<ceil_div(total, 256), 256, 0, s>>>(k, M, Pbar, ps, Qbar);
    LB_LAUNCH();
}

__global__ void fold_double_kernel(double* __restrict__ sk, double* __restrict__ sb, float* __restrict__ dk,
                                   float* __restrict__ db, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    dk[i] += (float)sk[i];
    db[i] += (float)sb[i];
    sk[i] = 0.0;
    sb[i] = 0.0;
}

void launch_fold_double(double* src_k, double* src_b, float* dst_k, float* dst_b, int64_t n, cudaStream_t s) {
    if (n == 0) return;
    fold_double_kernel<<<ceil_div(n, 256), 256, 0, s>>>(src_k, src_b, dst_k, dst_b, n);
    LB_LAUNCH();
}

__global__ void alpha_init_win_kernel(RowMap rows, WinGeo g, const float* __restrict__ init, int n,
                                      float* __restrict__ alpha) {
    const int nw = g.size();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    for (int r2 = blockIdx.y; r2 < 2 * rows.R; r2 += gridDim.y) {
        const int rr = r2 >= rows.R ? r2 - rows.R : r2;
        if (j >= nw) continue;
        int oy, ox;
        win_origin(g, rows.row_id[rr], oy, ox);
        const int nu = win_neuron(g, oy, ox, j);
        alpha[(size_t)r2 * nw + j] = nu >= 0 ? init[(size_t)rows.row_box[rr] * n + nu] : 0.f;
    }
}

void launch_alpha_init_win(const RowMap& rows, const WinGeo& g, const float* init_slope, int n, float* alpha,
                           cudaStream_t s) {
    if (rows.R == 0 || g.size() == 0) return;
    const dim3 grid(ceil_div(g.size(), 256), std::min(2 * rows.R, 65535));
    alpha_init_win_kernel<<<grid, 256, 0, s>>>(rows, g, init_slope, n, alpha);
    LB_LAUNCH();
}

}  // namespace lb200
