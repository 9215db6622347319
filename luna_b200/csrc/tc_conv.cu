// tc_conv.cu -- weights-stationary implicit-GEMM conv steps on tcgen05.
//
// One persistent CTA per SM walks (weight-row tile, pixel tile) pairs.
// Warp roles (12 warps, as in tc_gemm.cu):
//   warp 0      TMA producer: per K block the 128 x 32 weight tile (hi, lo)
//               and the shifted data box (raw fp32); TMEM allocation
//   warp 1      MMA issuer: per K=8 step three tcgen05.mma kind::tf32
//               (W_lo.X_hi, W_hi.X_lo, W_hi.X_hi) into a TMEM accumulator
//   warps 4-7   epilogue (lane = weight row, 16 pixels per TMEM load)
//   warps 8-11  split of the data box into (hi, lo) tf32 in place
// All waits are bounded; on expiry the CTA raises the error flag, drains
// what it issued and returns.
#include "tc_conv.cuh"
#include "tc_gemm.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>

namespace lb200 {

namespace {

using namespace tcx;

constexpr int NUM_THREADS = 384;
constexpr int WARP_TMA = 0, WARP_MMA = 1, EPI_WARP0 = 4, XF_WARP0 = 8;
constexpr int W_TILE_BYTES = 128 * 32 * 4;  // 16 KB
enum { KIND_FWD = 0, KIND_QBAR = 1 };

template <int BNMAX, int S, int KIND>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap twh,
                   const __grid_constant__ CUtensorMap twl, const __grid_constant__ TcConvPlan plan, int rows,
                   const __grid_constant__ TcConvFwd ef, const __grid_constant__ TcConvQbar eq, int* err) {
    constexpr int X_TILE_BYTES = BNMAX * 128;
    constexpr int STAGE_BYTES = 2 * W_TILE_BYTES + 2 * X_TILE_BYTES;
    constexpr uint32_t TMEM_COLS = (2 * BNMAX <= 32) ? 32 : (2 * BNMAX <= 64) ? 64 : (2 * BNMAX <= 128) ? 128
                                                        : (2 * BNMAX <= 256) ? 256 : 512;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + (size_t)S * STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* split = bars + S;
    uint64_t* empty = bars + 2 * S;
    uint64_t* tfull = bars + 3 * S;
    uint64_t* tempty = bars + 3 * S + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 4);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&split[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == WARP_TMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int N = plan.N;
    const int nyb = (plan.ny + plan.BY - 1) / plan.BY;
    const int n_tiles = ((rows + plan.BR - 1) / plan.BR) * nyb;
    const int m_tiles = (plan.m_total + 127) / 128;
    const int ntiles = n_tiles * m_tiles;
    const int nk = plan.nkb;
    const uint32_t box_bytes = (uint32_t)plan.BR * plan.BY * plan.BX * 128;

    auto w_hi = [&](int s) { return base + (size_t)s * STAGE_BYTES; };
    auto w_lo = [&](int s) { return base + (size_t)s * STAGE_BYTES + W_TILE_BYTES; };
    auto x_hi = [&](int s) { return base + (size_t)s * STAGE_BYTES + 2 * W_TILE_BYTES; };
    auto x_lo = [&](int s) { return base + (size_t)s * STAGE_BYTES + 2 * W_TILE_BYTES + X_TILE_BYTES; };

    if (warp == WARP_TMA) {
        if (lane == 0) {
            uint32_t g = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
                const int nt = t / m_tiles, mt = t % m_tiles;
                const int rb = nt / nyb, yb = nt % nyb;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % S;
                    const uint32_t ph = (g / S) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, abort, err)) break;
                    const TcConvTap tp = plan.kb[kb];
                    mbar_arrive_tx(&full[s], 2 * W_TILE_BYTES + box_bytes);
                    tma_load_2d(&twh, &full[s], w_hi(s), kb * 32, mt * 128);
                    tma_load_2d(&twl, &full[s], w_lo(s), kb * 32, mt * 128);
                    tma_load_5d(&tx, &full[s], x_hi(s), tp.c0, tp.dx, yb * plan.BY * plan.ds + tp.dy, tp.plane,
                                rb * plan.BR);
                }
            }
            if (*abort) {
                for (uint32_t q = (g > (uint32_t)S ? g - S : 0); q < g; ++q)
                    mbar_wait(&full[q % S], (q / S) & 1, abort, err, true);
            }
        }
    } else if (warp == WARP_MMA) {
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32(N);
            uint32_t g = 0, j = 0;
            bool issued = false;
            uint64_t* last_commit = nullptr;
            uint32_t last_phase = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++j) {
                const int acc = j & 1;
                const uint32_t aph = (j >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, abort, err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BNMAX);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % S;
                    const uint32_t ph = (g / S) & 1;
                    if (!mbar_wait(&split[s], ph, abort, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t dwh = desc_sw128(smem_u32(w_hi(s)));
                    const uint64_t dwl = desc_sw128(smem_u32(w_lo(s)));
                    const uint64_t dxh = desc_sw128(smem_u32(x_hi(s)));
                    const uint64_t dxl = desc_sw128(smem_u32(x_lo(s)));
#pragma unroll
                    for (int k8 = 0; k8 < 4; ++k8) {
                        const uint64_t off = (uint64_t)(k8 * 32) >> 4;
                        umma_tf32(d, dwl + off, dxh + off, idesc, (kb | k8) != 0);
                        umma_tf32(d, dwh + off, dxl + off, idesc, 1);
                        umma_tf32(d, dwh + off, dxh + off, idesc, 1);
                    }
                    umma_commit(&empty[s]);
                    issued = true;
                    last_commit = &empty[s];
                    last_phase = ph;
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
            }
            if (*abort && issued) mbar_wait(last_commit, last_phase, abort, err, true);
        }
    } else if (warp >= XF_WARP0) {
        const int xt = threadIdx.x - XF_WARP0 * 32;
        uint32_t g = 0;
        for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % S;
                const uint32_t ph = (g / S) & 1;
                if (!mbar_wait(&full[s], ph, abort, err)) {
                    ok = false;
                    break;
                }
                float4* hi = reinterpret_cast<float4*>(x_hi(s));
                float4* lo = reinterpret_cast<float4*>(x_lo(s));
                const int n4 = N * 8;
#pragma unroll 4
                for (int i = xt; i < n4; i += 128) {
                    const float4 x = hi[i];
                    float4 h, l;
                    h.x = rna_tf32(x.x); l.x = rna_tf32(x.x - h.x);
                    h.y = rna_tf32(x.y); l.y = rna_tf32(x.y - h.y);
                    h.z = rna_tf32(x.z); l.z = rna_tf32(x.z - h.z);
                    h.w = rna_tf32(x.w); l.w = rna_tf32(x.w - h.w);
                    hi[i] = h;
                    lo[i] = l;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&split[s]);
            }
            if (!ok) break;
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
        const int q = warp - EPI_WARP0;
        const int pix_per_row = plan.BY * plan.BX;
        uint32_t j = 0;
        for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++j) {
            const int nt = t / m_tiles, mt = t % m_tiles;
            const int rb = nt / nyb, yb = nt % nyb;
            const int acc = j & 1;
            const uint32_t aph = (j >> 1) & 1;
            if (!mbar_wait(&tfull[acc], aph, abort, err)) break;
            tc_fence_after();
            const int m = mt * 128 + q * 32 + lane;  // weight row of this thread
            const bool m_ok = m < plan.m_total;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BNMAX);
            if constexpr (KIND == KIND_FWD) {
                const int phase = m / ef.Ci, ci = m - (m / ef.Ci) * ef.Ci;
                const int py = phase / ef.s, px = phase - (phase / ef.s) * ef.s;
                const int nw = ef.out_h * ef.out_w * ef.Ci;
                // Output pixel of the first column of each 16-column chunk,
                // advanced column by column (warp-uniform).
                for (int c0 = 0; c0 < N; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + (uint32_t)c0, v);
                    int rl = c0 / pix_per_row, rem = c0 - rl * pix_per_row;
                    int yy = rem / plan.BX, xx = rem - yy * plan.BX;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = rb * plan.BR + rl;
                        const int ty = yb * plan.BY + yy;
                        const int vy = ef.s * (ty + ef.tlo_y) + py - ef.cy;
                        const int vx = ef.s * (xx + ef.tlo_x) + px - ef.cx;
                        if (m_ok && rl < plan.BR && r < rows && ty < plan.ny && (unsigned)vy < (unsigned)ef.out_h &&
                            (unsigned)vx < (unsigned)ef.out_w)
                            ef.P[(size_t)r * nw + (vy * ef.out_w + vx) * ef.Ci + ci] = v[i];
                        if (++xx == plan.BX) {
                            xx = 0;
                            if (++yy == plan.BY) {
                                yy = 0;
                                ++rl;
                            }
                        }
                    }
                }
            } else {
                const int co = m;
                const int nq = plan.ny * plan.nx * eq.Co;
                const float bco = (m_ok && eq.b) ? eq.b[co] : 0.f;
                for (int c0 = 0; c0 < N; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + (uint32_t)c0, v);
                    if (!m_ok) continue;
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {
                        const int n = c0 + i;
                        const int rl = n / pix_per_row, rem = n - rl * pix_per_row;
                        const int r = rb * plan.BR + rl;
                        if (n >= plan.BR * pix_per_row || r >= rows) break;
                        const int ty = yb * plan.BY + rem / plan.BX, tx = rem - (rem / plan.BX) * plan.BX;
                        if (ty >= plan.ny) continue;
                        eq.Qbar[(size_t)r * nq + (ty * eq.in_w + tx) * eq.Co + co] =
                            eq.b ? v[i] + eq.gseed[r] * bco : v[i];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == WARP_TMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
}

// ------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 conv_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

CUtensorMap map_2d(const float* p, int rows, int K, int box_rows) {
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = conv_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (weights) failed: " + std::to_string((int)r));
    return m;
}

CUtensorMap map_5d(const TcConvPlan& p) {
    CUtensorMap m;
    cuuint64_t dims[5] = {(cuuint64_t)p.C, (cuuint64_t)p.X, (cuuint64_t)p.Y, (cuuint64_t)p.P, (cuuint64_t)p.R};
    cuuint64_t strides[4];
    strides[0] = (cuuint64_t)p.C * 4;
    strides[1] = strides[0] * p.X;
    strides[2] = strides[1] * p.Y;
    strides[3] = strides[2] * p.P;
    // With ds > 1 the box traverses ds * BX x ds * BY pixels with element
    // stride ds, loading BX x BY of them (the same bytes as ds = 1).
    cuuint32_t box[5] = {32, (cuuint32_t)(p.BX * p.ds), (cuuint32_t)(p.BY * p.ds), 1, (cuuint32_t)p.BR};
    cuuint32_t estr[5] = {1, (cuuint32_t)p.ds, (cuuint32_t)p.ds, 1, 1};
    const CUresult r = conv_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(p.data), dims,
                                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (data) failed: " + std::to_string((int)r));
    return m;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        LB_CUDA(cudaGetDevice(&dev));
        LB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    }
    return n;
}

template <int BNMAX, int S, int KIND>
void run_conv(const TcConvPlan& p, int rows, const TcConvFwd& ef, const TcConvQbar& eq, cudaStream_t s) {
    constexpr int STAGE_BYTES = 2 * W_TILE_BYTES + 2 * BNMAX * 128;
    constexpr int SMEM = S * STAGE_BYTES + 1024 + 256;
    static bool configured = false;
    if (!configured) {
        LB_CUDA(cudaFuncSetAttribute(tc_conv_kernel<BNMAX, S, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        configured = true;
    }
    if (p.N > BNMAX || p.N % 16 != 0 || p.nkb <= 0 || p.nkb > TC_CONV_MAX_KB || p.ds < 1 || p.ds > 8 ||
        p.BX * p.ds > 256 || p.BY * p.ds > 256)
        throw std::invalid_argument("tc conv: bad tiling");
    const CUtensorMap tx = map_5d(p);
    const CUtensorMap twh = map_2d(p.w_hi, p.m_total, p.nkb * 32, 128);
    const CUtensorMap twl = map_2d(p.w_lo, p.m_total, p.nkb * 32, 128);
    const int nyb = (p.ny + p.BY - 1) / p.BY;
    const int64_t ntiles = (int64_t)((rows + p.BR - 1) / p.BR) * nyb * ((p.m_total + 127) / 128);
    const int grid = (int)std::min<int64_t>(ntiles, sm_count());
    tc_conv_kernel<BNMAX, S, KIND><<<grid, NUM_THREADS, SMEM, s>>>(tx, twh, twl, p, rows, ef, eq, tc_error_flag());
    LB_LAUNCH();
}

template <int KIND>
void dispatch_conv(const TcConvPlan& p, int rows, const TcConvFwd& ef, const TcConvQbar& eq, cudaStream_t s) {
    if (p.N > 128)
        run_conv<256, 2, KIND>(p, rows, ef, eq, s);
    else
        run_conv<128, 3, KIND>(p, rows, ef, eq, s);
}

}  // namespace

void tc_conv_set_wait_limit(long long wait_cycles) {
    LB_CUDA(cudaMemcpyToSymbol(tcx::g_wait_limit, &wait_cycles, sizeof(wait_cycles)));
}

bool tc_conv_supported(int data_C, int nx, int ds) {
    return data_C % 32 == 0 && data_C > 0 && nx >= 1 && ds >= 1 && ds <= 8 && nx * ds <= 256;
}

void tc_conv_tile(TcConvPlan& p, int rows) {
    p.BX = p.nx;
    // BY pixels rows of nx; the strided box spans BY * ds data rows (<= 256).
    p.BY = std::max(1, std::min(std::min(p.ny, 256 / p.nx), 256 / std::max(p.ds, 1)));
    p.BR = 1;
    if (p.BY >= p.ny) {
        p.BY = p.ny;
        p.BR = std::max(1, std::min(rows, 256 / (p.ny * p.nx)));
    }
    p.N = ((p.BR * p.BY * p.BX + 15) / 16) * 16;
}

void launch_tc_conv_fwd(const TcConvPlan& p, int rows, const TcConvFwd& e, cudaStream_t s) {
    if (rows == 0) return;
    dispatch_conv<KIND_FWD>(p, rows, e, TcConvQbar{}, s);
}

void launch_tc_conv_qbar(const TcConvPlan& p, int rows, const TcConvQbar& e, cudaStream_t s) {
    if (rows == 0) return;
    dispatch_conv<KIND_QBAR>(p, rows, TcConvFwd{}, e, s);
}

}  // namespace lb200
