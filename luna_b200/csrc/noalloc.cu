// noalloc.cu -- interval (IBP) bounds with no device allocation.
//
// Some callers cannot allocate device memory at the point where they need
// bounds: services that reserve all of their GPU memory up front and forbid
// allocation on the request path, hosts whose own memory manager owns every
// allocation on the device (another framework's caching allocator), and
// latency-critical loops that cannot afford cudaMalloc's implicit device
// synchronisation.  lb200_ibp_bounds_noalloc serves them: it computes the
// same IBP bounds as lb200_compute_bounds_device(..., LB200_METHOD_IBP, ...)
// but keeps the per-layer interval bounds in the fixed array below instead
// of engine-allocated buffers.  The caller still passes the input boxes, the
// specification and the output buffers.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds its 16 MiB until the process exits.  In host code its name
// is only a host-side stand-in, never a device address; the address is
// obtained per device with cudaGetSymbolAddress, with that device current,
// on the first call made on that device.  All calls share the array and it
// keeps the last call's contents; nothing in it needs to start at zero
// (every layer is fully written before it is read).  Calls whose work overlaps on the GPU
// (different streams, or different host threads) race on the array and
// must be serialised by the caller.
#include "handle.h"
#include "kernels.cuh"

#include <climits>
#include <mutex>
#include <string>

namespace {

// Capacity in floats: 4 Mi floats = 16 MiB.
constexpr int64_t kScratchFloats = int64_t(4) << 20;
__device__ __align__(256) float g_ibp_scratch[kScratchFloats];

std::mutex g_mu;
float* g_scratch_ptr[128] = {};

// Device address of g_ibp_scratch on the current device.
float* scratch_on_current_device() {
    int dev = 0;
    LB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 128) throw std::runtime_error("device index out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_ibp_scratch);
        if (e != cudaSuccess)
            throw std::runtime_error(std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e));
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" LB200_API int lb200_ibp_bounds_noalloc(lb200_model* model, const float* d_x_lower,
                                                  const float* d_x_upper, int64_t n_boxes, const float* d_C,
                                                  int64_t c_boxes, int64_t nspec, float* d_out_lb,
                                                  float* d_out_ub, void* stream) {
    if (!model || !model->m) return lb200::set_last_error("lb200_ibp_bounds_noalloc: null model");
    if (n_boxes <= 0 || nspec <= 0) return lb200::set_last_error("lb200_ibp_bounds_noalloc: empty batch");
    if (c_boxes != 1 && c_boxes != n_boxes)
        return lb200::set_last_error("lb200_ibp_bounds_noalloc: c_boxes must be 1 or n_boxes");
    if (!d_x_lower || !d_x_upper || !d_C || !d_out_lb || !d_out_ub)
        return lb200::set_last_error("lb200_ibp_bounds_noalloc: null buffer");
    // Sizes go to the kernels as int: keep n_boxes, nspec and their product in range.
    if (n_boxes > INT_MAX || nspec > INT_MAX || nspec > INT_MAX / n_boxes)
        return lb200::set_last_error("lb200_ibp_bounds_noalloc: n_boxes x nspec above 2^31 - 1");
    int prev_dev = -1;
    if (cudaGetDevice(&prev_dev) != cudaSuccess) prev_dev = -1;
    // The caller's current device is put back on every return path.
    struct Restore {
        int dev;
        ~Restore() {
            if (dev >= 0) cudaSetDevice(dev);
        }
    } restore{prev_dev};
    try {
        const lb200::Model& m = *model->m;
        if (!m.is_relu_mlp())
            return lb200::set_last_error(
                "lb200_ibp_bounds_noalloc: only Linear/ReLU networks (no conv, Sigmoid, Add or Sub on the input) are supported");
        const auto& L = m.layers();
        int64_t per_box = 0;
        for (const auto& layer : L) per_box += 2 * (int64_t)layer.n_out;
        // Compared by division: per_box * n_boxes may not fit in 64 bits.
        if (n_boxes > kScratchFloats / per_box)
            return lb200::set_last_error(
                "lb200_ibp_bounds_noalloc: " + std::to_string(n_boxes) + " boxes need " +
                (n_boxes <= INT64_MAX / per_box ? std::to_string(per_box * n_boxes) : std::string("> 2^63")) +
                " floats of scratch, above the fixed " +
                std::to_string(kScratchFloats) + " (at most " + std::to_string(kScratchFloats / per_box) +
                " boxes for this network)");
        LB_CUDA(cudaSetDevice(m.device()));
        float* scratch = scratch_on_current_device();
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const int B = (int)n_boxes;
        const float* in_l = d_x_lower;
        const float* in_u = d_x_upper;
        float* at = scratch;
        for (size_t k = 0; k < L.size(); ++k) {
            float* out_l = at;
            float* out_u = at + (size_t)B * L[k].n_out;
            lb200::launch_ibp_linear(L[k].W, L[k].b, in_l, in_u, out_l, out_u, B, L[k].n_in, L[k].n_out,
                                     k > 0, s);
            in_l = out_l;
            in_u = out_u;
            at = out_u + (size_t)B * L[k].n_out;
        }
        lb200::launch_ibp_spec(d_C, c_boxes == 1 ? 0 : 1, in_l, in_u, B, (int)nspec, L.back().n_out, d_out_lb,
                               d_out_ub, s);
        return 0;
    } catch (const std::exception& e) {
        return lb200::set_last_error(std::string("lb200_ibp_bounds_noalloc: ") + e.what());
    }
}
