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
// ceil(N / tc_block_n(N, pairs))).  With `pairs`, wide N that single CTAs
// would cut into 112-column tiles takes 224-column tiles on CTA pairs
// (tcgen05 cta_group::2, 256-row tiles): each SM of a pair stages half of the
// B tile and 128 rows of A.
int tc_block_n(int N, bool pairs);
int tc_tiles_n(int N, bool pairs);

// Split src into tf32 (hi, lo) with round-to-nearest: hi = rna(x),
// lo = rna(x - hi); n elements.
void launch_split_tf32(const float* src, float* hi, float* lo, int64_t n, cudaStream_t s);

// Device error flag written by a tensor-core kernel whose bounded waits ran
// out (0 = ok).  The engine checks it after each call.
int* tc_error_flag();
// Failure-detection test hook, on the current device: starve = 1 makes the
// tensor-core contraction producers issue no loads (their consumers' waits
// run out); wait_cycles > 0 sets the waits' limit (0: the default ~2 s).
void tc_set_test_fault(int starve, long long wait_cycles);
void tc_conv_set_wait_limit(long long wait_cycles);

// Adjoint contraction storing Qbar = A . B^T + g b_lin only; with
// e.seed_sign set the A operand is generated from the concretisation signs.
// split_acc: the cross terms of the split in a second TMEM accumulator
// (single-buffered accumulator, single CTAs).
void launch_tc_store_qbar(const float* A, const float* Bhi, const float* Blo, int M, int N, int K,
                          const EpiStoreQbar& e, bool pairs, bool split_acc, cudaStream_t s);

// Forward contraction whose A operand is the ReLU relaxation of P, formed in
// the kernel (BoundedReLUNode::boundBackward, dense A): Q = P+ s + P- k
// (lower side) or P+ k + P- s (upper side), s = alpha or the static lower
// slope.  P comes by TMA from `P` [M, K], or, when gather_W is set, is the
// row gather_W[row_id] (the one-hot start A . W of an intermediate start).
// The prologue also writes the row sums of the relaxation intercepts plus
// Q . b_lin (plus gather_b[row_id] when gathering) into bias_part[M].
struct TcPrologue {
    RowMap rows;
    ReluParams rp;                  // the ReLU below (rp.n == K)
    const float* P = nullptr;       // [M, K] (TMA) unless gather_W
    const float* alpha = nullptr;   // [M, K] or null (TMA)
    const float* b_lin = nullptr;   // [K]
    const float* gather_W = nullptr;
    const float* gather_b = nullptr;
    float* bias_part = nullptr;     // [M]
};
// One forward contraction.  A operand: the prologue's relaxation when
// pro.gather_W or pro.P is set, else the raw (already relaxed) A [M, K] by
// TMA.  Epilogue: the input concretisation when `conc` is set (partial sums
// per column tile), the next ReLU's relaxation when `fwd` is set (stores P
// and Q, partial sums per column tile), else a raw store of P into P_out.
void launch_tc_forward(const float* A, const TcPrologue& pro, const float* Bhi, const float* Blo, int M, int N,
                       int K, float* P_out, const EpiRelaxFwd* fwd, const EpiConcretize* conc, float* partial,
                       bool pairs, bool split_acc, cudaStream_t s);

}  // namespace lb200
