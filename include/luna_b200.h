/*
 * luna_b200.h -- C ABI of the B200 LiRPA bound-propagation engine.
 *
 * The engine computes IBP, CROWN and alpha-CROWN bounds for a batch of input
 * boxes on one GPU.  Every entry point returns an int status (0 = ok); the
 * message of the last failure on the calling thread is read with
 * lb200_last_error().  No C++ exception crosses this boundary.
 *
 * Ownership: the caller owns every host buffer it passes; the engine copies
 * weights to device memory at lb200_model_create() and owns all device
 * buffers it allocates.  A model handle is thread-compatible, not
 * thread-safe: one thread at a time may use a given handle.
 *
 * Reference interface replaced (Luna, paths within its project):
 *   - NLR::TorchModel(nodes, inputIndices, outputIndex, dependencies)
 *       src/engine/TorchModel.h:47-50           -> lb200_model_create
 *   - LunaConfiguration static result-affecting flags
 *       src/configuration/LunaConfiguration.cpp:22-66 -> lb200_options
 *   - TorchModel::compute_bounds(input_bounds, C, method, lower, upper)
 *       src/engine/TorchModel.h:97-103, TorchModel.cpp:653-698
 *                                                -> lb200_compute_bounds
 *   - Luna has one box per call (A is [spec, batch=1, features],
 *       src/engine/CROWNAnalysis.cpp:1106-1127); here one call bounds
 *       n_boxes independent boxes, each exactly as a fresh TorchModel
 *       would.
 */
#ifndef LUNA_B200_H
#define LUNA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LB200_API __attribute__((visibility("default")))
#else
#define LB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Node kinds.  The numbering is NLR::NodeType
 * (src/engine/nodes/BoundedTorchNode.h:37) so a front end that walks a Luna
 * graph can pass getNodeType() through unchanged. */
typedef enum {
    LB200_NODE_INPUT = 0,
    LB200_NODE_CONSTANT = 1,
    LB200_NODE_LINEAR = 2,
    LB200_NODE_RELU = 3,
    LB200_NODE_RESHAPE = 4,
    LB200_NODE_IDENTITY = 5,
    LB200_NODE_SUB = 6,
    LB200_NODE_FLATTEN = 7,
    LB200_NODE_ADD = 8,
    LB200_NODE_CONV = 9,
    LB200_NODE_BATCHNORM = 10,
    LB200_NODE_SIGMOID = 11,
    LB200_NODE_CONVTRANSPOSE = 12,
    LB200_NODE_CONCAT = 13,
    LB200_NODE_SLICE = 14
} lb200_node_type;

/* Analysis methods.  CROWN and ALPHA_CROWN are
 * LunaConfiguration::AnalysisMethod (src/configuration/LunaConfiguration.h:21-24);
 * IBP returns the interval bounds of the output node that Luna keeps in
 * CROWNAnalysis::getOutputIBPBounds (src/engine/CROWNAnalysis.cpp:1582-1589),
 * projected through the specification matrix C. */
enum {
    LB200_METHOD_IBP = 0,
    LB200_METHOD_CROWN = 1,
    LB200_METHOD_ALPHA_CROWN = 2
};

/* One node of the computation graph (one Bounded*Node).  Fields a node kind
 * does not use are ignored.  All pointers are host memory, fp32, row-major,
 * and only read during lb200_model_create().  Kinds the engine takes:
 * INPUT, LINEAR, CONV, CONVTRANSPOSE, BATCHNORM (after a LINEAR / CONV),
 * RELU, SIGMOID (on flat layers), ADD (two tensor producers: residual joins
 * of a ReLU output, directly or through a CONV), FLATTEN, IDENTITY,
 * RESHAPE (to a flat vector, as Luna's Reshape flattens), SUB with a
 * constant (on the input, or on a LINEAR / CONV output; a CONV's constant
 * uniform per channel), SLICE of a flat vector (of a LINEAR output, or
 * feeding LINEAR nodes), CONCAT along axis 1 of LINEAR outputs or of CONV
 * outputs that read the same producer with the same geometry; each of the
 * last four is rewritten into the same affine map over the kinds before it.
 * Other graphs are rejected by lb200_model_create with a message. */
typedef struct {
    int32_t type;          /* lb200_node_type */
    int32_t num_inputs;    /* number of producers (TorchModel dependencies) */
    int32_t inputs[4];     /* producer node indices, in dependency order */
    /* LINEAR: weight [out_features, in_features], bias [out_features] or NULL,
     * scale = ONNX Gemm alpha folded into the weight
     * (BoundedLinearNode.cpp:91-93). */
    int64_t in_features;
    int64_t out_features;
    float scale;
    const float* weight;
    const float* bias;
    /* Shape of this node's output as (C, H, W); a flat vector of n features
     * is (n, 1, 1).  Filled for every node. */
    int32_t out_shape[3];
    /* CONV / CONVTRANSPOSE geometry (square or rectangular kernels). */
    int32_t kernel[2];
    int32_t stride[2];
    int32_t padding[2];
    int32_t output_padding[2];
    /* BATCHNORM (eval mode): weight = gamma, bias = beta, plus running stats. */
    const float* running_mean;
    const float* running_var;
    float eps;
    /* SUB with one producer (BoundedSubNode::setConstantValue,
     * BoundedSubNode.h:54-57): constant [producer size] in Luna's flat (CHW)
     * order; constant_second = 1 for x - constant, 0 for constant - x. */
    const float* constant;
    int32_t constant_second;
    /* SLICE: BoundedSliceNode(start, end, axes, steps) (BoundedSliceNode.h:22)
     * with ONNX's conventions (negative start / end count from the end,
     * steps 1 or -1); CONCAT: BoundedConcatNode(axis, numInputs)
     * (BoundedConcatNode.h:22).  Axis 1 is the feature axis of a flat vector
     * or the channel axis of a (C, H, W) map. */
    int32_t axis;
    int64_t start;
    int64_t end;
    int64_t step;
} lb200_node_desc;

typedef struct {
    int32_t num_nodes;
    const lb200_node_desc* nodes;   /* indexed by node id */
    int32_t input_index;            /* TorchModel inputIndices[0] */
    int32_t output_index;           /* TorchModel outputIndex */
} lb200_graph_desc;

/* Result-affecting options, one field per LunaConfiguration flag
 * (src/configuration/LunaConfiguration.cpp:28-50).  lb200_options_default()
 * fills Luna's defaults. */
typedef struct {
    uint32_t alpha_iterations;        /* ALPHA_ITERATIONS = 20 */
    float alpha_lr;                   /* ALPHA_LR = 0.5 */
    float alpha_lr_decay;             /* ALPHA_LR_DECAY = 0.98 */
    uint32_t early_stop_patience;     /* EARLY_STOP_PATIENCE = 10 */
    float start_save_best;            /* START_SAVE_BEST = 0.5 */
    int32_t stabilize_intermediate_bounds;  /* STABILIZE_INTERMEDIATE_BOUNDS = 1 */
    int32_t recompute_intermediate_bounds;  /* RECOMPUTE_INTERMEDIATE_BOUNDS = 1 */
    int32_t optimize_lower;           /* OPTIMIZE_LOWER = 1 */
    int32_t optimize_upper;           /* OPTIMIZE_UPPER = 0 */
    int32_t stop_crown_on_verified;   /* STOP_CROWN_ON_VERIFIED = 1 */
    int32_t stop_alpha_on_verified;   /* STOP_ALPHA_ON_VERIFIED = 1 */
    int32_t enable_first_linear_ibp;  /* ENABLE_FIRST_LINEAR_IBP = 1 */
    int32_t use_patches_mode;         /* USE_PATCHES_MODE = 1 */
} lb200_options;

/* Per-call statistics. */
typedef struct {
    double ms_total;          /* wall time of the call on the host */
    double ms_device;         /* CUDA-event time of the device work */
    int64_t kernel_launches;  /* kernels this call launched */
    int64_t backward_rows;    /* A-matrix rows (both sides) propagated */
    double algorithmic_flops; /* 2*M*N*K summed over real rows, contractions */
    int32_t alpha_iterations_run; /* max over boxes */
    /* Filled when profiling is on (lb200_set_profiling): CUDA-event time of
     * the A.W contraction kernels, their launches and their 2*M*N*K. */
    double ms_contractions;
    int64_t contraction_launches;
    double contraction_flops;
} lb200_stats;

typedef struct lb200_model lb200_model;

/* Fill *opt with Luna's defaults (LunaConfiguration.cpp:28-50). */
LB200_API int lb200_options_default(lb200_options* opt);

/* Build a model on CUDA device `device`.  Replaces
 * TorchModel(nodes, inputIndices, outputIndex, dependencies)
 * (src/engine/TorchModel.h:47-50, TorchModel.cpp:23-64). */
LB200_API int lb200_model_create(const lb200_graph_desc* graph, int device, lb200_model** out);

/* Set the result-affecting options (the LunaConfiguration globals that
 * TorchModel::compute_bounds reads, TorchModel.cpp:668-670,683-684). */
LB200_API int lb200_set_options(lb200_model* model, const lb200_options* opt);

/* Bound n_boxes input boxes.  Replaces TorchModel::compute_bounds
 * (src/engine/TorchModel.cpp:653-698) called once per box on a fresh model.
 *   x_lower, x_upper : [n_boxes, n_in] host, the flat input box per box
 *   C                : [c_boxes, nspec, n_out] host; c_boxes is 1 (shared)
 *                      or n_boxes (one specification per box)
 *   thresholds       : [nspec] host or NULL.  With thresholds, a box one of
 *                      whose lower bounds exceeds its row's threshold
 *                      counts as verified (TorchModel::isSpecVerified,
 *                      TorchModel.cpp:616-651, for a conjunction; see
 *                      lb200_compute_property for disjunctions) and the
 *                      STOP_*_ON_VERIFIED options apply; without them
 *                      nothing is ever verified, as in Luna after
 *                      setSpecificationMatrix.
 *   out_lb, out_ub   : [n_boxes, nspec] host
 *   stats            : may be NULL. */
LB200_API int lb200_compute_bounds(lb200_model* model, int method,
                         const float* x_lower, const float* x_upper, int64_t n_boxes,
                         const float* C, int64_t c_boxes, int64_t nspec,
                         const float* thresholds, int bound_lower, int bound_upper,
                         float* out_lb, float* out_ub, lb200_stats* stats);

/* As lb200_compute_bounds, with every array already in device memory of the
 * model's GPU; the work is ordered on `stream` (a cudaStream_t, or NULL for
 * the legacy default stream) and the call returns once it has completed. */
LB200_API int lb200_compute_bounds_device(lb200_model* model, int method,
                                const float* d_x_lower, const float* d_x_upper, int64_t n_boxes,
                                const float* d_C, int64_t c_boxes, int64_t nspec,
                                const float* d_thresholds, int bound_lower, int bound_upper,
                                float* d_out_lb, float* d_out_ub, void* stream,
                                lb200_stats* stats);

/* Time every A.W contraction kernel with CUDA events on the launching stream
 * (on != 0) so lb200_stats reports ms_contractions.  Off by default.  Luna
 * has no counterpart: it exists for roofline measurement. */
LB200_API int lb200_set_profiling(lb200_model* model, int on);

/* Contraction path: 0 (default) uses the tcgen05 tensor cores with 3xTF32
 * split precision wherever the shape allows (N a multiple of 16, K of 4),
 * with 224-column tiles on CTA pairs (cta_group::2) for wide N, the SIMT fp32
 * kernel elsewhere, and the adjoint contractions accumulating the split's
 * cross terms apart from its main term; 1 uses the SIMT fp32 kernel
 * everywhere; 2 the tensor cores on single CTAs only; 3 the tensor cores
 * for the forward contractions and the SIMT kernel for the adjoint ones;
 * 4 as 0 without the separate cross-term accumulation; 5 as 0 with it in
 * the forward contractions too (1-5 for cross-checking).  Luna has no
 * counterpart. */
LB200_API int lb200_set_contraction_path(lb200_model* model, int path);

/* Warm start, as branch-and-bound hands each sub-domain its parent's state
 * (TorchModel::getState / TorchModel::loadState, src/engine/TorchModel.h:123-135,
 * and AlphaCROWNAnalysis::seedAlphas, src/engine/AlphaCROWNAnalysis.cpp:971-997).
 * With keep != 0, every later alpha-CROWN call retains its boxes' final
 * alphas (the ones getState returns) and their creation sets; keep == 0
 * drops them.  lb200_set_warm_parents(model, parent, n) then makes the NEXT
 * call (alpha-CROWN, n boxes, one chunk) start box b from retained box
 * parent[b]: per (ReLU, start) the parent's alphas are reused, row by row,
 * when the start has as many rows for box b as it had for the parent, and
 * created afresh otherwise; the reused alphas are their own best alphas, so
 * restoring the best alphas leaves them as optimised; no CROWN
 * initialisation pass.  parent[b] == -1 bounds box b afresh.  Intermediate
 * bounds are recomputed (Luna's RECOMPUTE_INTERMEDIATE_BOUNDS default).
 * Networks with Sigmoid, OPTIMIZE_UPPER, specification thresholds and calls
 * split into chunks are refused (an error, not a fresh run).  Both return 0, or nonzero with lb200_last_error set. */
LB200_API int lb200_set_warm_start(lb200_model* model, int keep);
LB200_API int lb200_set_warm_parents(lb200_model* model, const int64_t* parent, int64_t n);
/* The alpha part of TorchModel::getState (src/engine/TorchModel.cpp:995-1014)
 * for one retained box: the alphas of activation `level` (1-based, in
 * topological order) for start `start` (the pre-activation of level `start`,
 * 2 <= start < K, or the output, start == K, for a network of K affine
 * layers), both sides, as [2][rows][cols] floats (side 0 lower, 1 upper;
 * rows = that start's rows for the box; cols = the activation's width: every
 * neuron, where Luna keeps only the creation set's); creation_set (may be
 * NULL) receives [cols] bytes, 1 for the neurons the alpha was created for.
 * *rows and *cols are always set; out is written only when
 * cap >= 2 * rows * cols (out NULL: sizes only). */
LB200_API int lb200_warm_alpha(lb200_model* model, int level, int start, int64_t box, float* out, int64_t cap,
                               int64_t* rows, int64_t* cols, uint8_t* creation_set);

/* IBP bounds of n_boxes boxes without allocating any device memory, for
 * Linear/ReLU networks (models with convs, Sigmoid or Add are rejected): the
 * same result as lb200_compute_bounds_device(..., LB200_METHOD_IBP, ...),
 * for callers that cannot call cudaMalloc where they need bounds (a service
 * that reserves its GPU memory up front and forbids allocation on the
 * request path, or a host whose own memory manager owns every allocation).
 * The per-layer interval bounds live in a fixed 16 MiB __device__ array
 * held by every GPU that loads this library until the process exits;
 * batches needing more (n_boxes * 2 * sum of Linear output widths floats
 * above 4 Mi) are rejected with an error, as are n_boxes * nspec above
 * 2^31 - 1.  Work is enqueued on `stream` (a stream of the model's device)
 * and the call returns without waiting; the caller's current device is left
 * as it was.  The first call on a device resolves the array's address on
 * that device (cudaGetSymbolAddress), so make that first call before any
 * stream capture begins.  All calls share the
 * array, so calls that overlap on the GPU race and must be serialised by
 * the caller.  No counterpart in the reference. */
LB200_API int lb200_ibp_bounds_noalloc(lb200_model* model, const float* d_x_lower,
                                       const float* d_x_upper, int64_t n_boxes, const float* d_C,
                                       int64_t c_boxes, int64_t nspec, float* d_out_lb,
                                       float* d_out_ub, void* stream);

/* Failure-detection test hook for the tensor-core kernels' bounded waits,
 * on CUDA device `device`.  starve = 1 makes the contraction producers
 * announce their TMA loads but issue none, so every consumer's wait runs
 * out: the kernels raise the device error flag and return, and the call that
 * launched them returns non-zero ("a bounded wait expired") with the
 * context still usable.  wait_cycles > 0 sets the waits' limit in SM clock
 * cycles (0: the default, about 2 s).  (0, 0) restores normal operation.
 * Luna has no counterpart (it runs no device waits). */
LB200_API int lb200_test_set_contraction_fault(int device, int starve, int64_t wait_cycles);

/* Copy the intermediate (pre-activation) bounds of the last call into host
 * buffers: for every node that feeds a ReLU, in node-id order, [n_boxes,
 * size] lower then upper.  Mirrors TorchModel::getState().allBounds
 * (src/engine/TorchModel.cpp:975-1014).  *count receives the total floats
 * per side; pass NULL buffers to query it. */
LB200_API int lb200_get_intermediate_bounds(lb200_model* model, float* lower, float* upper, int64_t* count);

/* ---- multi-GPU: box sharding over NCCL ------------------------------------
 * Luna bounds one box per call and has no distributed path; boxes share only
 * the read-only weights.  N ranks, one process per GPU, each bound a
 * contiguous share of a batch and exchange only the final bounds (one NCCL
 * all-gather).  NCCL is resolved at run time from the process's
 * libnccl.so.2, so a caller may pass its own ncclComm_t as `comm`. */

/* [begin, end) of n boxes for `rank` of `world` (shares differ by at most one). */
LB200_API int lb200_shard_range(int rank, int world, int64_t n, int64_t* begin, int64_t* end);

/* A 128-byte ncclUniqueId made on one rank and shared with the others by the
 * caller; lb200_nccl_comm_create then joins the communicator on `device`
 * (blocks until all `world` ranks have joined) and runs one all-gather so
 * that NCCL's peer connections exist before the first lb200_shard_run: a
 * communicator passed in by the caller should have run a collective of its
 * own first, since NCCL sets up connections on first use and that setup
 * waits on the host, outside lb200_shard_run's bounded wait. */
LB200_API int lb200_nccl_unique_id(uint8_t id[128]);
LB200_API int lb200_nccl_comm_create(const uint8_t id[128], int rank, int world, int device, void** comm);
LB200_API int lb200_nccl_comm_destroy(void* comm);

/* Every rank passes the whole batch (host buffers, as lb200_compute_bounds);
 * rank r bounds its share lb200_shard_range(r, world, n_boxes) and all
 * ranks receive the bounds of every box in out_lb / out_ub [n_boxes, nspec].
 * The wait for the gather is bounded by timeout_ms (60 s when <= 0): when it
 * expires, or NCCL reports an asynchronous error, the communicator is
 * aborted (ncclCommAbort releases it: the caller must neither use nor
 * destroy it afterwards) and an error naming the abort returned; the model
 * stays usable.  stats covers this rank's share. */
LB200_API int lb200_shard_run(lb200_model* model, void* comm, int rank, int world, int method,
                              const float* x_lower, const float* x_upper, int64_t n_boxes,
                              const float* C, int64_t c_boxes, int64_t nspec,
                              float* out_lb, float* out_ub, int timeout_ms, lb200_stats* stats);

/* Host only (no GPU is touched): check the graph as lb200_model_create does
 * and describe the engine's plan for it as JSON -- every level (node, map
 * shape, activation, main edge, skip edges) and every backward start (the
 * concretisation form Luna's CPU path uses for it and the row window at each
 * level below it).  *needed receives the length including the terminator;
 * buf may be NULL to query it.  No counterpart in the reference. */
LB200_API int lb200_describe_plan(const lb200_graph_desc* graph, const lb200_options* opt, char* buf, size_t len,
                                  size_t* needed);

/* ---- VNN-LIB properties ---------------------------------------------------
 * A property is an input box over the variables X_i and output constraints
 * over Y_j that describe the counterexample region: "C.y <= thresholds"
 * for a conjunction of rows, or a disjunction (OR) of such conjunctions
 * (branches).  The property is UNSAT (verified) when the bounds show that
 * region unreachable.  Replaces VnnLibInputParser::parseInputBounds /
 * parseOutputConstraints (src/input_parsers/VnnLibInputParser.cpp:335-372,
 * 917-928), OutputConstraintSet::toCMatrix (OutputConstraint.cpp:71-173) and
 * the CLI's evaluatePropertyStatus (src/engine/LunaMain.cpp:60-135). */
typedef struct lb200_property lb200_property;

typedef enum {
    LB200_STATUS_UNKNOWN = 0, /* the bounds decide nothing */
    LB200_STATUS_UNSAT = 1,   /* verified: the counterexample region is unreachable */
    LB200_STATUS_SAT = 2      /* every point of the box is a counterexample */
} lb200_status;

typedef struct lb200_property_info {
    int64_t n_in, n_out; /* the sizes the property was parsed for */
    int64_t nspec;       /* rows of C; 0 when the text has no usable output constraints */
    int32_t n_branches;  /* OR branches; 0 for a plain conjunction */
    int32_t spec_dropped; /* 1 when output constraints were present but failed to convert */
    char spec_error[256]; /* why, when spec_dropped */
} lb200_property_info;

/* Parse VNN-LIB text (the bytes of a .vnnlib file) for a network with n_in
 * inputs and n_out outputs, as TorchModel(onnxPath, vnnlibPath) does
 * (src/engine/TorchModelOnnxFactory.cpp:89-192): lines are trimmed, blank and
 * ';' comment lines dropped, the rest joined; X_i bounds missing from the
 * text are -inf / +inf; X_i with i >= n_in are ignored.  A malformed input
 * bound fails the call.  Output constraints that fail to convert (a Y_j with
 * j >= n_out, a bad number) leave the property without a specification, as
 * Luna continues without them; info.spec_dropped says so. */
LB200_API int lb200_property_parse(const char* text, int64_t len, int64_t n_in, int64_t n_out,
                                   lb200_property** out);
LB200_API int lb200_property_get_info(const lb200_property* prop, lb200_property_info* info);
/* lower, upper: [n_in] each. */
LB200_API int lb200_property_input_box(const lb200_property* prop, float* lower, float* upper);
/* C: [nspec, n_out]; thresholds: [nspec]; branch_of_row: [nspec] (all 0 for
 * a conjunction).  Any of them may be NULL. */
LB200_API int lb200_property_spec(const lb200_property* prop, float* C, float* thresholds, int32_t* branch_of_row);
LB200_API void lb200_property_free(lb200_property* prop);

/* The verdict of each of n_boxes boxes from the bounds of its nspec rows
 * (host arrays; lb, ub [n_boxes, nspec]); n_branches == 0 for a
 * conjunction, else branch_of_row [nspec] gives each row's branch in
 * [0, n_branches).  status: [n_boxes] lb200_status values. */
LB200_API int lb200_property_status(const float* lb, const float* ub, int64_t n_boxes, int64_t nspec,
                                    const float* thresholds, const int32_t* branch_of_row, int32_t n_branches,
                                    int32_t* status);
/* As lb200_property_status with every array in device memory of the current
 * CUDA device, one thread per box, ordered on `stream`; returns without
 * waiting. */
LB200_API int lb200_property_status_device(const float* d_lb, const float* d_ub, int64_t n_boxes, int64_t nspec,
                                           const float* d_thresholds, const int32_t* d_branch_of_row,
                                           int32_t n_branches, int32_t* d_status, void* stream);

/* Bound n_boxes boxes against a property, as the Luna CLI does for one
 * (TorchModel(onnx, vnnlib) then compute_bounds(inputBounds, nullptr,
 * method) then evaluatePropertyStatus, LunaMain.cpp:240-330): C, thresholds
 * and branches come from the property and are shared by every box, so the
 * STOP_CROWN_ON_VERIFIED / STOP_ALPHA_ON_VERIFIED options apply per box.
 * x_lower / x_upper [n_boxes, n_in] host (sub-boxes of a split, say), or
 * both NULL with n_boxes == 1 for the property's own input box.  out_lb,
 * out_ub: [n_boxes, rows] host with rows = nspec, or n_out (raw output
 * bounds, status UNKNOWN) when the property has no specification.
 * status: [n_boxes] or NULL. */
LB200_API int lb200_compute_property(lb200_model* model, int method, const lb200_property* prop,
                                     const float* x_lower, const float* x_upper, int64_t n_boxes,
                                     float* out_lb, float* out_ub, int32_t* status, lb200_stats* stats);

/* As lb200_compute_property with the boxes and the results in device memory
 * of the model's GPU (d_x_lower, d_x_upper [n_boxes, n_in]; d_out_lb,
 * d_out_ub [n_boxes, rows]; d_status [n_boxes] or NULL); the property's
 * specification is copied to the device on each call.  The work is ordered
 * on `stream` (a cudaStream_t, or NULL for the legacy default stream) and
 * the call returns once it has completed. */
LB200_API int lb200_compute_property_device(lb200_model* model, int method, const lb200_property* prop,
                                            const float* d_x_lower, const float* d_x_upper, int64_t n_boxes,
                                            float* d_out_lb, float* d_out_ub, int32_t* d_status, void* stream,
                                            lb200_stats* stats);

/* Copy the last error message of this thread into buf (always terminated). */
LB200_API int lb200_last_error(char* buf, size_t len);

/* Release the model and every device buffer it owns. */
LB200_API void lb200_model_destroy(lb200_model* model);

#ifdef __cplusplus
}
#endif

#endif /* LUNA_B200_H */
