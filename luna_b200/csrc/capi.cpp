// capi.cpp -- extern "C" entry points declared in include/luna_b200.h.
// Every entry point catches all exceptions and reports them through
// lb200_last_error(); nothing is thrown across the boundary.
#include "handle.h"
#include "tc_gemm.cuh"

#include <cstring>
#include <exception>
#include <string>

namespace {
thread_local std::string g_last_error;

int fail(const std::string& msg) {
    g_last_error = msg;
    return 1;
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    } catch (...) {
        return fail("unknown error");
    }
}
}  // namespace

int lb200::set_last_error(const std::string& msg) { return fail(msg); }

extern "C" {

int lb200_options_default(lb200_options* o) {
    if (!o) return fail("lb200_options_default: null options");
    o->alpha_iterations = 20;
    o->alpha_lr = 0.5f;
    o->alpha_lr_decay = 0.98f;
    o->early_stop_patience = 10;
    o->start_save_best = 0.5f;
    o->stabilize_intermediate_bounds = 1;
    o->recompute_intermediate_bounds = 1;
    o->optimize_lower = 1;
    o->optimize_upper = 0;
    o->stop_crown_on_verified = 1;
    o->stop_alpha_on_verified = 1;
    o->enable_first_linear_ibp = 1;
    o->use_patches_mode = 1;
    return 0;
}

int lb200_model_create(const lb200_graph_desc* graph, int device, lb200_model** out) {
    if (!out) return fail("lb200_model_create: null output handle");
    *out = nullptr;
    return guarded([&] {
        auto* h = new lb200_model;
        try {
            h->m = new lb200::Model(graph, device);
            LB_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
        } catch (...) {
            delete h->m;
            delete h;
            throw;
        }
        *out = h;
    });
}

int lb200_set_options(lb200_model* model, const lb200_options* opt) {
    if (!model || !opt) return fail("lb200_set_options: null argument");
    if (!opt->recompute_intermediate_bounds)
        return fail("lb200_set_options: recompute_intermediate_bounds = 0 is not supported");
    model->m->set_options(*opt);
    return 0;
}

int lb200_set_profiling(lb200_model* model, int on) {
    if (!model) return fail("lb200_set_profiling: null model");
    model->m->set_profiling(on != 0);
    return 0;
}

int lb200_set_contraction_path(lb200_model* model, int path) {
    if (!model) return fail("lb200_set_contraction_path: null model");
    if (path < 0 || path > 5) return fail("lb200_set_contraction_path: path must be 0 to 5");
    model->m->set_force_simt(path == 1);
    model->m->set_pairs(path != 2);
    model->m->set_simt_adjoint(path == 3);
    model->m->set_split_acc(path != 4, path == 5);
    return 0;
}

int lb200_set_warm_start(lb200_model* model, int keep) {
    if (!model) return fail("lb200_set_warm_start: null model");
    model->m->set_warm_keep(keep != 0);
    return 0;
}

int lb200_set_warm_parents(lb200_model* model, const int64_t* parent, int64_t n) {
    if (!model) return fail("lb200_set_warm_parents: null model");
    return guarded([&] { model->m->set_warm_parents(parent, n); });
}

int lb200_warm_alpha(lb200_model* model, int level, int start, int64_t box, float* out, int64_t cap,
                     int64_t* rows, int64_t* cols, uint8_t* creation_set) {
    if (!model || !rows || !cols) return fail("lb200_warm_alpha: null argument");
    return guarded([&] { model->m->warm_alpha(level, start, box, out, cap, rows, cols, creation_set); });
}

int lb200_compute_bounds_device(lb200_model* model, int method, const float* d_x_lower,
                                const float* d_x_upper, int64_t n_boxes, const float* d_C,
                                int64_t c_boxes, int64_t nspec, const float* d_thresholds,
                                int bound_lower, int bound_upper, float* d_out_lb, float* d_out_ub,
                                void* stream, lb200_stats* stats) {
    if (!model) return fail("lb200_compute_bounds_device: null model");
    if (n_boxes > 0 && (!d_x_lower || !d_x_upper || !d_C || !d_out_lb || !d_out_ub))
        return fail("lb200_compute_bounds_device: null buffer");
    return guarded([&] {
        model->m->compute(method, d_x_lower, d_x_upper, n_boxes, d_C, c_boxes, nspec, d_thresholds,
                          bound_lower != 0, bound_upper != 0, d_out_lb, d_out_ub,
                          static_cast<cudaStream_t>(stream), stats);
    });
}

int lb200_compute_bounds(lb200_model* model, int method, const float* x_lower, const float* x_upper,
                         int64_t n_boxes, const float* C, int64_t c_boxes, int64_t nspec,
                         const float* thresholds, int bound_lower, int bound_upper, float* out_lb,
                         float* out_ub, lb200_stats* stats) {
    if (!model) return fail("lb200_compute_bounds: null model");
    if (n_boxes > 0 && (!x_lower || !x_upper || !C || !out_lb || !out_ub))
        return fail("lb200_compute_bounds: null buffer");
    return guarded([&] {
        lb200::Model& m = *model->m;
        LB_CUDA(cudaSetDevice(m.device()));
        cudaStream_t s = model->stream;
        const size_t nx = (size_t)n_boxes * m.n_in();
        const size_t nc = (size_t)c_boxes * nspec * m.n_out();
        const size_t no = (size_t)n_boxes * nspec;
        float* dxl = m.staging("io_xl", nx);
        float* dxu = m.staging("io_xu", nx);
        float* dC = m.staging("io_C", nc);
        float* dlb = m.staging("io_lb", no);
        float* dub = m.staging("io_ub", no);
        float* dthr = thresholds ? m.staging("io_thr", nspec) : nullptr;
        LB_CUDA(cudaMemcpyAsync(dxl, x_lower, nx * 4, cudaMemcpyHostToDevice, s));
        LB_CUDA(cudaMemcpyAsync(dxu, x_upper, nx * 4, cudaMemcpyHostToDevice, s));
        LB_CUDA(cudaMemcpyAsync(dC, C, nc * 4, cudaMemcpyHostToDevice, s));
        if (dthr) LB_CUDA(cudaMemcpyAsync(dthr, thresholds, nspec * 4, cudaMemcpyHostToDevice, s));
        m.compute(method, dxl, dxu, n_boxes, dC, c_boxes, nspec, dthr, bound_lower != 0,
                  bound_upper != 0, dlb, dub, s, stats);
        LB_CUDA(cudaMemcpyAsync(out_lb, dlb, no * 4, cudaMemcpyDeviceToHost, s));
        LB_CUDA(cudaMemcpyAsync(out_ub, dub, no * 4, cudaMemcpyDeviceToHost, s));
        LB_CUDA(cudaStreamSynchronize(s));
    });
}

int lb200_get_intermediate_bounds(lb200_model* model, float* lower, float* upper, int64_t* count) {
    if (!model || !count) return fail("lb200_get_intermediate_bounds: null argument");
    return guarded([&] {
        *count = model->m->intermediate_count();
        if (lower && upper) model->m->copy_intermediate(lower, upper);
    });
}

int lb200_describe_plan(const lb200_graph_desc* graph, const lb200_options* opt, char* buf, size_t len,
                        size_t* needed) {
    return guarded([&] {
        lb200::Model m(graph, 0, /*on_device=*/false);
        if (opt) m.set_options(*opt);
        const std::string j = m.describe();
        if (needed) *needed = j.size() + 1;
        if (buf && len) {
            std::strncpy(buf, j.c_str(), len - 1);
            buf[len - 1] = '\0';
        }
    });
}

int lb200_test_set_contraction_fault(int device, int starve, int64_t wait_cycles) {
    return guarded([&] {
        if (wait_cycles < 0) throw std::invalid_argument("wait_cycles must be >= 0");
        LB_CUDA(cudaSetDevice(device));
        lb200::tc_set_test_fault(starve ? 1 : 0, (long long)wait_cycles);
    });
}

int lb200_last_error(char* buf, size_t len) {
    if (!buf || len == 0) return 1;
    std::strncpy(buf, g_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
    return 0;
}

void lb200_model_destroy(lb200_model* model) {
    if (!model) return;
    try {
        if (model->m) cudaSetDevice(model->m->device());
        if (model->stream) cudaStreamDestroy(model->stream);
        delete model->m;
    } catch (...) {
    }
    delete model;
}

}  // extern "C"
