// shard.cpp -- multi-GPU box sharding over NCCL (extern "C" entry points
// declared in include/luna_b200.h).
//
// Luna bounds one box per TorchModel::compute_bounds call and has no
// distributed path (CROWNAnalysis.cpp:1106-1127): boxes share only the
// read-only weights.  N ranks, one process per GPU, each bound a contiguous
// share of the batch; the one exchange is an all-gather of the final
// [boxes, nspec] bounds.  NCCL is resolved at run time from the process's
// libnccl.so.2 (the copy a framework already loaded, else the system's), so
// the library links no NCCL and a caller's own ncclComm_t can be passed in.
#include "handle.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    std::string load_error;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.load_error = std::string("libnccl.so.2 could not be loaded: ") + dlerror();
            return;
        }
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p && api.load_error.empty()) api.load_error = std::string("NCCL symbol missing: ") + name;
            return p;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
        api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    });
    if (!api.load_error.empty()) throw std::runtime_error(api.load_error);
    return api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + nccl().error_string(r));
}

// Contiguous [begin, end) of n boxes for `rank`; sizes differ by at most one.
void range_of(int rank, int world, int64_t n, int64_t& begin, int64_t& end) {
    const int64_t base = n / world, extra = n % world;
    begin = rank * base + std::min<int64_t>(rank, extra);
    end = begin + base + (rank < extra ? 1 : 0);
}

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        return lb200::set_last_error(e.what());
    } catch (...) {
        return lb200::set_last_error("unknown error");
    }
}

}  // namespace

extern "C" {

int lb200_shard_range(int rank, int world, int64_t n, int64_t* begin, int64_t* end) {
    if (!begin || !end) return lb200::set_last_error("lb200_shard_range: null output");
    if (world <= 0 || rank < 0 || rank >= world || n < 0) return lb200::set_last_error("lb200_shard_range: bad rank");
    range_of(rank, world, n, *begin, *end);
    return 0;
}

int lb200_nccl_unique_id(uint8_t id[128]) {
    if (!id) return lb200::set_last_error("lb200_nccl_unique_id: null id");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    return guard([&] {
        ncclUniqueId u;
        nccl_check(nccl().get_unique_id(&u), "ncclGetUniqueId");
        std::memcpy(id, &u, 128);
    });
}

int lb200_nccl_comm_create(const uint8_t id[128], int rank, int world, int device, void** comm) {
    if (!id || !comm) return lb200::set_last_error("lb200_nccl_comm_create: null argument");
    if (world <= 0 || rank < 0 || rank >= world) return lb200::set_last_error("lb200_nccl_comm_create: bad rank");
    *comm = nullptr;
    return guard([&] {
        LB_CUDA(cudaSetDevice(device));
        ncclUniqueId u;
        std::memcpy(&u, id, 128);
        ncclComm_t c = nullptr;
        nccl_check(nccl().comm_init_rank(&c, world, u, rank), "ncclCommInitRank");
        // NCCL sets up a collective's peer connections on its first use, and
        // that setup waits on the host for every peer.  One all-gather now,
        // while every rank is known to be here, makes it happen at creation,
        // so that a later gather whose peer never arrives only waits on the
        // device, where lb200_shard_run's bounded wait can abort it.
        cudaStream_t s = nullptr;
        float* buf = nullptr;
        try {
            LB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
            LB_CUDA(cudaMalloc(&buf, sizeof(float) * (size_t)(world + 1)));
            LB_CUDA(cudaMemsetAsync(buf, 0, sizeof(float) * (size_t)(world + 1), s));
            nccl_check(nccl().all_gather(buf + world, buf, 1, ncclFloat32, c, s), "ncclAllGather (connection setup)");
            LB_CUDA(cudaStreamSynchronize(s));
        } catch (...) {
            if (buf) cudaFree(buf);
            if (s) cudaStreamDestroy(s);
            nccl().comm_abort(c);
            throw;
        }
        LB_CUDA(cudaFree(buf));
        LB_CUDA(cudaStreamDestroy(s));
        *comm = c;
    });
}

int lb200_nccl_comm_destroy(void* comm) {
    if (!comm) return 0;
    return guard([&] { nccl_check(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy"); });
}

int lb200_shard_run(lb200_model* model, void* comm, int rank, int world, int method, const float* x_lower,
                    const float* x_upper, int64_t n_boxes, const float* C, int64_t c_boxes, int64_t nspec,
                    float* out_lb, float* out_ub, int timeout_ms, lb200_stats* stats) {
    if (!model || !comm) return lb200::set_last_error("lb200_shard_run: null model or communicator");
    if (world <= 0 || rank < 0 || rank >= world) return lb200::set_last_error("lb200_shard_run: bad rank");
    if (n_boxes < 0 || nspec <= 0 || (c_boxes != 1 && c_boxes != n_boxes))
        return lb200::set_last_error("lb200_shard_run: bad sizes");
    if (n_boxes > 0 && (!x_lower || !x_upper || !C || !out_lb || !out_ub))
        return lb200::set_last_error("lb200_shard_run: null buffer");
    return guard([&] {
        lb200::Model& m = *model->m;
        const int64_t n_in = m.n_in(), n_out = m.n_out();
        int64_t a = 0, b = 0;
        range_of(rank, world, n_boxes, a, b);
        // This rank's share, bounded into its rows of the output.
        if (b > a) {
            const float* Cs = C + (c_boxes == 1 ? 0 : a * nspec * n_out);
            if (lb200_compute_bounds(model, method, x_lower + a * n_in, x_upper + a * n_in, b - a, Cs,
                                     c_boxes == 1 ? 1 : b - a, nspec, nullptr, 1, 1, out_lb + a * nspec,
                                     out_ub + a * nspec, stats) != 0) {
                char msg[512];
                lb200_last_error(msg, sizeof msg);
                throw std::runtime_error(msg);
            }
        }
        // All-gather [2, width, nspec] per rank (shares padded to the largest).
        int64_t width = 0;
        for (int r = 0; r < world; ++r) {
            int64_t ra, rb;
            range_of(r, world, n_boxes, ra, rb);
            width = std::max(width, rb - ra);
        }
        const size_t per = (size_t)2 * width * nspec;
        if (per == 0) return;
        LB_CUDA(cudaSetDevice(m.device()));
        cudaStream_t s = model->stream;
        float* send = m.staging("shard_send", per);
        float* recv = m.staging("shard_recv", per * world);
        LB_CUDA(cudaMemsetAsync(send, 0, per * 4, s));
        const size_t mine = (size_t)(b - a) * nspec * 4;
        if (mine) {
            LB_CUDA(cudaMemcpyAsync(send, out_lb + a * nspec, mine, cudaMemcpyHostToDevice, s));
            LB_CUDA(cudaMemcpyAsync(send + (size_t)width * nspec, out_ub + a * nspec, mine, cudaMemcpyHostToDevice, s));
        }
        const NcclApi& api = nccl();
        ncclComm_t c = static_cast<ncclComm_t>(comm);
        nccl_check(api.all_gather(send, recv, per, ncclFloat32, c, s), "ncclAllGather");
        // Bounded wait: a rank that never reaches the gather must not leave
        // this one (and its GPU) waiting; abort the communicator instead.
        const auto t0 = std::chrono::steady_clock::now();
        while (true) {
            const cudaError_t q = cudaStreamQuery(s);
            if (q == cudaSuccess) break;
            if (q != cudaErrorNotReady) LB_CUDA(q);
            ncclResult_t ar = ncclSuccess;
            nccl_check(api.comm_get_async_error(c, &ar), "ncclCommGetAsyncError");
            const double ms =
                std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            if (ar != ncclSuccess || ms > (timeout_ms > 0 ? timeout_ms : 60000)) {
                api.comm_abort(c);
                throw std::runtime_error(ar != ncclSuccess
                                             ? std::string("bound gather failed (") + api.error_string(ar) +
                                                   "); the communicator was aborted"
                                             : "bound gather timed out; the communicator was aborted");
            }
            std::this_thread::sleep_for(std::chrono::microseconds(200));
        }
        std::vector<float> host(per * world);
        LB_CUDA(cudaMemcpy(host.data(), recv, host.size() * 4, cudaMemcpyDeviceToHost));
        for (int r = 0; r < world; ++r) {
            if (r == rank) continue;
            int64_t ra, rb;
            range_of(r, world, n_boxes, ra, rb);
            const float* blk = host.data() + per * r;
            std::memcpy(out_lb + ra * nspec, blk, (size_t)(rb - ra) * nspec * 4);
            std::memcpy(out_ub + ra * nspec, blk + (size_t)width * nspec, (size_t)(rb - ra) * nspec * 4);
        }
    });
}

}  // extern "C"
