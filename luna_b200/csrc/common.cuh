// common.cuh -- shared helpers of the luna_b200 CUDA engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace lb200 {

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void check_cuda(cudaError_t e, const char* what, const char* file, int line) {
    if (e != cudaSuccess)
        throw CudaError(std::string(what) + " failed at " + file + ":" + std::to_string(line) +
                        ": " + cudaGetErrorString(e));
}

// Kernels launched by this thread since it last reset the counter.
inline int64_t& launch_counter() {
    static thread_local int64_t n = 0;
    return n;
}

inline void count_launch(const char* file, int line) {
    check_cuda(cudaGetLastError(), "kernel launch", file, line);
    ++launch_counter();
}

#define LB_CUDA(x) ::lb200::check_cuda((x), #x, __FILE__, __LINE__)
#define LB_LAUNCH() ::lb200::count_launch(__FILE__, __LINE__)

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// One torch::optim::Adam step (betas 0.9 / 0.999, eps 1e-8, no weight decay)
// followed by AlphaCROWNAnalysis::clipAlphaParameters' clamp to [0, 1]:
//   m = m*b1 + (1-b1) g;  v = v*b2 + (1-b2) g g;
//   a += -step * m / (sqrt(v) / sqrt(bc2) + eps),  step = lr / bc1.
__device__ __forceinline__ float adam_clip_update(float a, float g, float& m, float& v, float step,
                                                  float bc2_sqrt) {
    m = m * 0.9f + 0.1f * g;
    v = v * 0.999f + 0.001f * g * g;
    const float denom = sqrtf(v) / bc2_sqrt + 1e-8f;
    a = a + (-step) * m / denom;
    return fminf(fmaxf(a, 0.f), 1.f);
}

// Per-(box, neuron) relaxation flags of one ReLU.
enum : uint8_t {
    RF_USE_ALPHA = 1,   // lower slope comes from the alpha tensor
    RF_UNSTABLE = 2,    // lb < 0 < ub now: k_up / b_up carry gradient to the bounds
    RF_ASET = 4,        // in the alpha creation set: only these alphas ever take a
                        // nonzero Adam step (the others keep m = v = 0)
};

}  // namespace lb200
