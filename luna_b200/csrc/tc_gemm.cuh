// tc_gemm.cuh -- sm_100a tensor-core contraction (tcgen05 + TMEM + TMA) with
// fp32-accurate 3xTF32 split precision and the engine's fused epilogues.
//
// P = A . B^T with A [M, K] fp32 row-major and B [N, K] fp32 row-major
// (both K-major).  B is given as a (hi, lo) pair split once at model
// creation; A is loaded raw by TMA and split into (hi, lo) in shared memory.
// D = A_lo B_hi + A_hi B_lo + A_hi B_hi accumulates in fp32 in TMEM.
#pragma once

#include "kernels.cuh"

namespace lb200 {

// True when the shape can use the tensor-core path (TMA needs 16-byte row
// strides; the MMA needs N a multiple of 16).
bool tc_supported(int M, int N, int K);
// Column tile of the tensor-core path for N (its partial-sum tile count is
// ceil(N / tc_block_n(N))).
int tc_block_n(int N);
int tc_tiles_n(int N);

// Split src into tf32 (hi, lo) with round-to-nearest: hi = rna(x),
// lo = rna(x - hi); n elements.
void launch_split_tf32(const float* src, float* hi, float* lo, int64_t n, cudaStream_t s);

// Device error flag written by a tensor-core kernel whose bounded waits ran
// out (0 = ok).  The engine checks it after each call.
int* tc_error_flag();

void launch_tc_relax_fwd(const float* A, const float* Bhi, const float* Blo, int M, int N, int K,
                         const EpiRelaxFwd& e, float* partial, cudaStream_t s);
void launch_tc_concretize(const float* A, const float* Bhi, const float* Blo, int M, int N, int K,
                          const EpiConcretize& e, float* partial, cudaStream_t s);
// Adjoint: the k_up / b_up slots are per (32-row group, virtual box).
void launch_tc_relax_adj(const float* A, const float* Bhi, const float* Blo, int M, int N, int K,
                         const EpiRelaxAdj& e, cudaStream_t s);
// Adjoint contraction storing Qbar = A . B^T + g b_lin only; with
// e.seed_sign set the A operand is generated from the concretisation signs.
void launch_tc_store_qbar(const float* A, const float* Bhi, const float* Blo, int M, int N, int K,
                          const EpiStoreQbar& e, cudaStream_t s);

}  // namespace lb200
