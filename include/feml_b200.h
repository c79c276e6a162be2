/*
 * feml_b200.h -- C ABI of libfeml_b200.so, a B200 (sm_100a) backend for
 * feml's mul_mat / mul_mat_id path.
 *
 * Conventions
 *  - Every call returns int status: FB_OK (0) or an FB_ERR_* code; the
 *    message of the last failure on the calling thread is returned by
 *    feml_b200_last_error(). No C++ exception or abort crosses this boundary
 *    (the reference's zero-panic contract, feml-core/src/backend.rs:80-122).
 *  - Enum values are the discriminants of the reference enums: DType
 *    (feml-core/src/dtype.rs:14-35), Op (feml-core/src/op.rs:12-43),
 *    BufferUsage (feml-core/src/backend.rs:52-57).
 *  - Tensor layout is ggml's: ne[] element counts, nb[] byte strides,
 *    nb[0] = type_size, nb[1] = row bytes (feml-core/src/layout.rs:32-48).
 *  - "stream" arguments are cudaStream_t passed as void* (NULL = the legacy
 *    default stream).
 */
#ifndef FEML_B200_H
#define FEML_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* every declaration below is exported even when the library is built with
 * -fvisibility=hidden */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes ------------------------------------------------------ */
#define FB_OK 0
#define FB_ERR_INVALID 1     /* bad argument, unknown handle, range outside a buffer */
#define FB_ERR_UNSUPPORTED 2 /* op / dtype / shape not supported by this backend */
#define FB_ERR_SHAPE 3       /* shape or layout mismatch (reference ErrorKind::Shape) */
#define FB_ERR_CUDA 4        /* CUDA runtime error */
#define FB_ERR_DEVICE 5      /* error reported by a kernel (e.g. mul_mat_id id out of range) */
#define FB_ERR_NO_DEVICE 6   /* no usable sm_100 device */

/* ---- enums (reference discriminants) ----------------------------------- */
enum fb_dtype {
    FB_I8 = 0, FB_I16, FB_I32, FB_I64, FB_F16, FB_F32, FB_F64,
    FB_Q4_0, FB_Q4_1, FB_Q5_0, FB_Q5_1, FB_Q8_0, FB_Q8_1,
    FB_Q2_K, FB_Q3_K, FB_Q4_K, FB_Q5_K, FB_Q6_K, FB_Q8_K,
    FB_DTYPE_COUNT
};

enum fb_op {
    FB_OP_NONE = 0, FB_OP_VIEW, FB_OP_MUL, FB_OP_ADD, FB_OP_MUL_MAT, FB_OP_MUL_MAT_ID,
    FB_OP_RMS_NORM, FB_OP_SOFTMAX, FB_OP_ROPE, FB_OP_SILU, FB_OP_GET_ROWS, FB_OP_CONCAT,
    FB_OP_COPY, FB_OP_DIAG_MASK_INF, FB_OP_SCALE
};

enum fb_usage { FB_USAGE_WEIGHTS = 0, FB_USAGE_COMPUTE = 1 };

/* TensorFlags bits, feml-core/src/tensor.rs:48-68 */
#define FB_FLAG_INPUT 1u
#define FB_FLAG_OUTPUT 2u
#define FB_FLAG_WEIGHT 4u

/* ---- plan mirror: repr(C) image of feml_core::plan::GraphPlan ----------
 * (feml-core/src/plan.rs:15-45). A Rust caller fills these from its
 * GraphPlan; op_params carries the inline Op payload (MulMatId:
 * [0] = n_experts, [1] = n_selected). */
#define FB_MAX_SRC 4
typedef struct {
    uint32_t id;
    int32_t op;
    uint32_t op_params[2];
    int32_t n_srcs;
    int32_t srcs[FB_MAX_SRC]; /* indices into fb_plan.tensors */
    int32_t buffer;           /* index into fb_plan.buffers */
    uint64_t offset;          /* byte offset within the buffer */
    int32_t dtype;
    uint32_t flags;
    int64_t ne[4];
    uint64_t nb[4];
} fb_plan_tensor;

typedef struct {
    uint32_t handle;
    uint64_t size;
    int32_t usage;
} fb_plan_buffer;

typedef struct {
    uint64_t uid;
    const fb_plan_tensor *tensors;
    int64_t n_tensors;
    const int64_t *nodes; /* indices into tensors, execution order */
    int64_t n_nodes;
    const fb_plan_buffer *buffers;
    int64_t n_buffers;
} fb_plan;

/* ---- generic backend vtable: C image of `&dyn Backend` -----------------
 * (feml-core/src/backend.rs:86-122). GraphBuilder::compile below drives any
 * backend through this table; feml_b200_backend_vtable() fills one for the
 * B200 backend. */
typedef struct {
    void *ctx;
    const char *(*name)(void *ctx);
    int (*create_buffer)(void *ctx, uint64_t size, int32_t usage, uint32_t *handle);
    int (*release_buffer)(void *ctx, uint32_t handle);
    int (*write)(void *ctx, uint32_t handle, uint64_t offset, const void *src, uint64_t n);
    int (*read)(void *ctx, uint32_t handle, uint64_t offset, void *dst, uint64_t n);
    int (*fill)(void *ctx, uint32_t handle, uint64_t offset, uint8_t value, uint64_t n);
    int (*synchronize)(void *ctx);
    int (*graph_compute)(void *ctx, const fb_plan *plan);
    int (*supports_op)(void *ctx, int32_t op, const int32_t *src_dtypes, int32_t n);
    /* Optional (may be NULL; no counterpart in the Rust trait): called by
     * fb_graph_compile once the plan's buffers exist, so the backend can size
     * its intermediates and prepare the plan's launches at compile time
     * instead of on the first graph_compute. */
    int (*prepare_plan)(void *ctx, const fb_plan *plan);
} fb_backend_vtable;

const char *feml_b200_last_error(void);
const char *feml_b200_version(void);

/* ======================================================================== */
/* 1. Backend (the drop-in boundary).                                       */
/* ======================================================================== */
typedef struct fb_backend fb_backend;

typedef struct {
    char name[256];
    uint64_t memory_total;
    uint64_t memory_free;
    int32_t cc_major, cc_minor;
    int32_t sm_count;
    int32_t device_type; /* feml-core DeviceType: 1 = Gpu */
    int32_t async_compute, host_buffer, events;
} fb_device_info;

/* BackendRegistrar::device_count / score (feml-core/src/backend.rs:157-165;
 * CUDA registrar scores 1000, feml-cuda/src/device.rs:118-120; this backend
 * reports 2000 when an sm_100 device is present, else 0). */
int feml_b200_device_count(int32_t *count);
int feml_b200_registrar_score(uint32_t *score);
/* BackendDevice::info (feml-core/src/backend.rs:130-131). */
int feml_b200_device_info(int32_t device, fb_device_info *info);

/* BackendDevice::init_backend (feml-core/src/backend.rs:133-134): one
 * backend = one device + one CUDA stream. */
int feml_b200_open(int32_t device, fb_backend **out);
int feml_b200_close(fb_backend *b);
/* Backend::name -> "B200". */
const char *feml_b200_name(fb_backend *b);
/* Backend::create_buffer, zero-initialised (backend.rs:90-92). */
int feml_b200_create_buffer(fb_backend *b, uint64_t size, int32_t usage, uint32_t *handle);
/* Backend::release_buffer (backend.rs:94-95). */
int feml_b200_release_buffer(fb_backend *b, uint32_t handle);
/* Backend::write / read: blocking; the byte range must lie inside the
 * buffer or FB_ERR_INVALID is returned and nothing is written
 * (backend.rs:97-103). A write of at most 1 MiB returns once the bytes are
 * copied into the backend's pinned staging area; the device copy is queued
 * on the backend stream ahead of every later read, fill and graph_compute
 * (the caller may reuse `src` at once; a copy error surfaces at the next
 * synchronize or read). */
int feml_b200_write(fb_backend *b, uint32_t handle, uint64_t offset, const void *src, uint64_t n);
int feml_b200_read(fb_backend *b, uint32_t handle, uint64_t offset, void *dst, uint64_t n);
/* Backend::fill (backend.rs:105-106), asynchronous like the reference CUDA
 * fill kernel (feml-cuda/src/kernels.cu:124-133). */
int feml_b200_fill(fb_backend *b, uint32_t handle, uint64_t offset, uint8_t value, uint64_t n);
/* Backend::synchronize (backend.rs:108-109). Also reports, once, any error
 * a kernel recorded since the last call (FB_ERR_DEVICE). */
int feml_b200_synchronize(fb_backend *b);
/* Backend::supports_op (backend.rs:117-121): 1 = supported, 0 = not.
 * MulMat: src0 in {F32, Q8_0, Q4_0, Q4_K}, src1 = F32.
 * MulMatId: src0 in the same set, src1 = F32, src2 = I32. */
int feml_b200_supports_op(fb_backend *b, int32_t op, const int32_t *src_dtypes, int32_t n);
/* Backend::graph_compute (backend.rs:111-114): enqueues the plan on the
 * backend stream and returns. The first call of a plan may grow the scratch
 * arena (with a stream synchronize) and captures the plan's CUDA graph (see
 * feml_b200_set_plan_graphs); later calls of the same plan allocate nothing
 * and do not synchronize. */
int feml_b200_graph_compute(fb_backend *b, const fb_plan *plan);
/* Nodes of `plan` that graph_compute folds into a neighbouring kernel
 * instead of running them: an rms_norm feeding only decode mul_mats (inside
 * their activation quantization), and the bias add / SiLU after a mul_mat
 * (inside its epilogue: a mul_mat whose output is read only by an add with
 * an M-float bias vector and/or a silu, each intermediate read once, not an
 * output and computed by the next node). The reference plans both fusions
 * for compile time (docs/DESIGN.md:250-251). */
int feml_b200_plan_fused_nodes(fb_backend *b, const fb_plan *plan, int64_t *count);

/* Fill a vtable bound to `b` (for compile() and other generic callers). */
int feml_b200_backend_vtable(fb_backend *b, fb_backend_vtable *vt);

/* Prepare a compiled plan for execution (fb_graph_compile does this through
 * the vtable; a caller that compiles elsewhere, such as the Rust
 * GraphBuilder::compile of graph.rs:349-442, calls it once after compile):
 * the scratch arena grows to the plan's largest node and the plan's launches
 * are captured into a CUDA graph. graph_compute of a prepared plan then
 * allocates nothing, from its first call on (docs/backend-guide.md:22). */
int feml_b200_prepare_plan(fb_backend *b, const fb_plan *plan);

/* Interop: device address of a buffer and the backend's CUDA stream. */
int feml_b200_buffer_device_ptr(fb_backend *b, uint32_t handle, void **ptr, uint64_t *size);
int feml_b200_stream(fb_backend *b, void **stream);
/* Bytes of device scratch the backend holds for mul_mat/mul_mat_id
 * intermediates (sized when a Compute buffer is created; grown at most once
 * more, at the first graph_compute of a plan that needs more;
 * reserve_scratch sizes it ahead of time). */
int feml_b200_scratch_bytes(fb_backend *b, uint64_t *bytes);
int feml_b200_reserve_scratch(fb_backend *b, uint64_t bytes);
/* Device allocations (cudaMalloc of buffers and of the scratch arena) this
 * backend has made so far: the zero-allocation contract of graph_compute
 * (docs/backend-guide.md:22; the reference checks it with a counting global
 * allocator, feml-cpu/tests/cpu_integration.rs:11-34,230-251) is observable
 * as this count staying unchanged across repeated graph_compute calls. */
int feml_b200_device_allocations(fb_backend *b, uint64_t *count);
/* Plan graphs (GraphPlan.uid is the reference's plan-caching hook,
 * feml-core/src/plan.rs:38-39, graph.rs:335-347): graph_compute replays a
 * CUDA graph of a plan's launches from its second call on (captured, not
 * executed, during the first). Enabled by default; disabling (or enabling)
 * synchronizes the stream and drops the cached graphs. plan_graphs reports
 * how many plans are cached and how many of those replay a graph. */
int feml_b200_set_plan_graphs(fb_backend *b, int32_t enable);
int feml_b200_plan_graphs(fb_backend *b, int64_t *cached, int64_t *replayable);

/* ======================================================================== */
/* 2. Graph builder / planner mirror (C++ restatement of feml-core's        */
/*    GraphBuilder -> compile -> GraphPlan, feml-core/src/graph.rs,         */
/*    planner.rs, plan.rs), used by C/C++/Python callers without Rust.      */
/* ======================================================================== */
typedef struct fb_graph fb_graph;
typedef struct fb_compiled_plan fb_compiled_plan;

int fb_graph_new(fb_graph **out);
void fb_graph_free(fb_graph *g);
/* GraphBuilder::input / weight (graph.rs:67-87). */
int fb_graph_input(fb_graph *g, const char *name, int32_t dtype, const int64_t *dims, int32_t rank, uint32_t *id);
int fb_graph_weight(fb_graph *g, const char *name, int32_t dtype, const int64_t *dims, int32_t rank, uint32_t *id);
/* GraphBuilder::view (graph.rs:89-108). */
int fb_graph_view(fb_graph *g, uint32_t src, uint64_t offset, const int64_t *dims, int32_t rank, uint32_t *id);
/* GraphBuilder::mul / add (graph.rs:110-120); built for planner parity,
 * not executed by this backend (supports_op = 0). */
int fb_graph_mul(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id);
int fb_graph_add(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id);
int fb_graph_silu(fb_graph *g, uint32_t x, uint32_t *id);
/* GraphBuilder::rms_norm (graph.rs:140-142): y = x / sqrt(mean(x^2) + eps)
 * along ne0; eps in op_params[0] (f32 bits). */
int fb_graph_rms_norm(fb_graph *g, uint32_t x, float eps, uint32_t *id);
int fb_graph_copy(fb_graph *g, uint32_t x, uint32_t *id);
/* GraphBuilder::mul_mat (graph.rs:122-138), relaxed: src0 in {F32, Q8_0,
 * Q4_0, Q4_K, Q5_K, Q6_K}, src1 F32, output F32 [ne1(a), ne1(b)], ne0(a) % block == 0
 * (mul_mat_id: F32, Q8_0, Q4_0, Q4_K). */
int fb_graph_mul_mat(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id);
/* GraphBuilder::mul_mat_id (graph.rs:215-250), ggml semantics: weights
 * [K, M, E], x [K, N], ids I32 [n_selected, N], output F32
 * [M, n_selected, N]; out[:, s, t] = W[:, :, ids[s, t]]^T x[:, t]. */
int fb_graph_mul_mat_id(fb_graph *g, uint32_t w, uint32_t x, uint32_t ids, uint32_t n_selected, uint32_t *id);
/* GraphBuilder::mark_output (graph.rs:57-65). */
int fb_graph_mark_output(fb_graph *g, uint32_t id);
/* Tensor metadata: dtype, ne[4], nb[4], flags, op. */
int fb_graph_tensor_info(fb_graph *g, uint32_t id, int32_t *dtype, int64_t *ne, uint64_t *nb, uint32_t *flags, int32_t *op);
/* GraphBuilder::compile (graph.rs:349-442) against any backend vtable. */
int fb_graph_compile(fb_graph *g, const fb_backend_vtable *backend, fb_compiled_plan **out);

const fb_plan *fb_plan_get(fb_compiled_plan *p);
/* GraphPlan::find (plan.rs:54-56): index into tensors, or -1. */
int64_t fb_plan_find(fb_compiled_plan *p, uint32_t id);
/* GraphPlan::write_tensor / read_tensor (plan.rs:77-115): n must equal the
 * tensor's nbytes. */
int fb_plan_write_tensor(fb_compiled_plan *p, const fb_backend_vtable *backend, uint32_t id, const void *src, uint64_t n);
int fb_plan_read_tensor(fb_compiled_plan *p, const fb_backend_vtable *backend, uint32_t id, void *dst, uint64_t n);
/* GraphPlan::release (plan.rs:68-73). */
int fb_plan_release(fb_compiled_plan *p, const fb_backend_vtable *backend);
void fb_plan_free(fb_compiled_plan *p);

/* Planner-only entry (feml-core/src/planner.rs:156-261) for planner parity
 * tests: tensors described by (id, dtype, ne, flags, op, srcs, view_src,
 * view_offset); `order` indexes them; out receives per-tensor (kind, offset),
 * kind 0 = Weights, 1 = Compute. */
typedef struct {
    uint32_t id;
    int32_t dtype;
    int64_t ne[4];
    int32_t rank;
    uint32_t flags;
    int32_t op;
    int32_t n_srcs;
    uint32_t srcs[FB_MAX_SRC]; /* tensor ids */
    uint32_t view_src;         /* 0 = not a view */
    uint64_t view_offset;
} fb_planner_tensor;

int fb_planner_plan(const fb_planner_tensor *tensors, int64_t n, const int64_t *order, int64_t n_order,
                    int32_t *kinds, uint64_t *offsets, uint64_t *weights_size, uint64_t *compute_size);

/* Layout helpers (layout.rs:32-60, dtype.rs:105-116). */
int fb_layout_new(int32_t dtype, const int64_t *dims, int32_t rank, uint64_t *nb);
int fb_layout_nbytes(int32_t dtype, const int64_t *ne, const uint64_t *nb, uint64_t *nbytes);
int fb_dtype_traits(int32_t dtype, int64_t *block_size, int64_t *type_size, int32_t *quantized);

/* ======================================================================== */
/* 3. Kernel-level entry points on device pointers (what graph_compute     */
/*    launches). All asynchronous on `stream`.                              */
/* ======================================================================== */

/* Quantize `rows` rows of `k` f32 (row r at x + r*x_row_stride bytes) into
 * ggml blocks of `dtype` (FB_Q8_0, FB_Q4_0, FB_Q4_K), row r at
 * y + r*row_size(dtype, k). FB_Q8_0 on activations is quantize_row_q8_0:
 * d = f16(amax/127), q = round-half-away(x * (1/d)). The Q4_K scheme is this
 * library's deterministic single-pass quantizer. */
int feml_b200_quantize(int32_t dtype, const void *x, uint64_t x_row_stride, void *y, int64_t rows, int64_t k,
                       void *stream);

/* Workspace bytes feml_b200_mul_mat needs for this shape (0 when the
 * activation quantisation is fused into the kernel). */
int feml_b200_mul_mat_workspace(int32_t wtype, int64_t K, int64_t M, int64_t N, uint64_t *bytes);

/* mul_mat, ggml semantics (feml-cpu/src/ops/mul_mat.rs:14-58):
 *   dst[m*4 + n*dst_nb1] = sum_k W[k, m] * X[k, n]
 * W: wtype blocks, row m at w + m*w_nb1; X: f32, column n at x + n*x_nb1;
 * quantized weights are multiplied against the Q8_0-quantized activations:
 * int32 per-block sums on the decode GEMVs (N <= 8) and on the Q4_K GEMM
 * when K % 512 != 0; the Q8_0 / Q4_0 / Q4_K (K % 512 == 0) GEMM (N > 8)
 * multiplies the dequantized values, each split exactly into two f16, with
 * f32 accumulation (Q4_K: d * (sc * q) split, and -dmin * m against the
 * activation block sums). That GEMM needs every dequantized weight within
 * the f16 range (|d| <= 511.75 for Q8_0, <= 8188 for Q4_0; for Q4_K
 * |d| <= 65504/945 and |dmin| <= 65504/63; quantized model weights stay far
 * below). Under
 * graph_compute a larger block scale sets bit 3 of the backend's status
 * word, which synchronize reports as FB_ERR_DEVICE; this entry point has no
 * status word, and such a scale shows as non-finite outputs. dst must not
 * overlap w or x. */
int feml_b200_mul_mat(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *dst,
                      uint64_t dst_nb1, int64_t K, int64_t M, int64_t N, void *workspace, uint64_t workspace_bytes,
                      void *stream);

/* Number of kernel launches one feml_b200_mul_mat of this shape enqueues
 * (16-byte aligned operands): the decode GEMV, the activation quantizer and
 * GEMM, and a split-K reduction when the GEMM splits K. For benchmarks that
 * count the kernels of a timed region. */
int feml_b200_mul_mat_launches(int32_t wtype, int64_t K, int64_t M, int64_t N, int32_t *count);

/* feml_b200_mul_mat without a workspace argument: the scratch is a fixed
 * 16 MiB device array inside this library (one per device), so the call
 * allocates nothing. No counterpart in the reference (its backends allocate
 * per call or plan every byte ahead). Same kernels and results as
 * feml_b200_mul_mat. The first call on each device looks the array up
 * (cudaGetSymbolAddress, with that device current) and should come before
 * any stream capture. All calls on a device share the array: calls whose
 * kernels can overlap (unordered streams) race; calls on one stream are
 * safe. Nothing in it needs to start at zero. Shapes whose scratch
 * (feml_b200_mul_mat_workspace) exceeds feml_b200_mul_mat_noalloc_limit()
 * bytes return FB_ERR_UNSUPPORTED without queuing work; arguments are
 * checked first as feml_b200_mul_mat checks them (negative dimensions:
 * FB_ERR_INVALID). The array is device memory of the library's own module:
 * under lazy module loading (the CUDA 12 default) a device holds it from the
 * first call made there; with CUDA_MODULE_LOADING=EAGER every context the
 * process creates holds it from creation. */
int feml_b200_mul_mat_noalloc(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *dst,
                              uint64_t dst_nb1, int64_t K, int64_t M, int64_t N, void *stream);
uint64_t feml_b200_mul_mat_noalloc_limit(void);

int feml_b200_mul_mat_id_workspace(int32_t wtype, int64_t K, int64_t M, int64_t N, int64_t n_selected,
                                   int64_t n_experts, uint64_t *bytes);

/* mul_mat_id, ggml semantics: expert e's weight rows at w + e*w_nb2 + m*w_nb1;
 * x column t at x + t*x_nb1; ids[s + t*ids_nb1/4] selects the expert of slot
 * (s, t); dst column (s, t) at dst + s*dst_nb1 + t*dst_nb2. Slots with an id
 * outside [0, n_experts) produce zeros and set bit 1 of *status (device
 * int32, may be NULL). */
int feml_b200_mul_mat_id(int32_t wtype, const void *w, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                         const void *x, uint64_t x_nb1, const int32_t *ids, uint64_t ids_nb1, int64_t n_selected,
                         void *dst, uint64_t dst_nb1, uint64_t dst_nb2, int64_t K, int64_t M, int64_t N,
                         void *workspace, uint64_t workspace_bytes, int32_t *status, void *stream);

/* Row-sharded decode mul_mat with the all-gather fused into the kernel (no
 * counterpart in the reference, which has no multi-device code). This rank
 * holds weight rows [row0, row0 + M) of the full matrix. Each rank owns two
 * output buffers used alternately by step; peer_dst0[r] / peer_dst1[r] are
 * rank r's buffers already offset to row0 (device pointers valid on this
 * device: its own memory or a CUDA IPC mapping of the peer's), column n at
 * + n*dst_nb1. Every output value is stored into every rank's buffer of this
 * step (buffer (*epoch + 1) & 1) over NVLink; when the grid is done each
 * peer_flags[r] (a uint32 in rank r's memory) is raised by one. `counter` is
 * a zeroed uint32 of this rank used by the grid (left at zero) and `epoch`
 * this rank's completed-step count (advanced by feml_b200_peer_wait).
 * Quantized weights, N <= 8 and N*K <= 16384 (the fused-quantization GEMV).
 * Both calls take only device state, so a step can be captured in a CUDA
 * graph and replayed. */
int feml_b200_mul_mat_peer(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1,
                           void *const *peer_dst0, void *const *peer_dst1, uint32_t *const *peer_flags,
                           int32_t n_peers, uint64_t dst_nb1, uint32_t *counter, const uint32_t *epoch, int64_t K,
                           int64_t M, int64_t N, int32_t *status, void *stream);

/* Map another process's device allocation (a 64-byte cudaIpcMemHandle_t)
 * into the current device's context with peer access enabled, so kernels on
 * this device can load and store it over NVLink; *base is the start of the
 * allocation. No counterpart in the reference. */
int feml_b200_ipc_open(const void *handle, uint64_t handle_bytes, void **base);
/* The IPC handle (64 bytes) of the device allocation holding ptr and ptr's
 * byte offset in it. */
int feml_b200_ipc_export(const void *ptr, void *handle, uint64_t handle_bytes, uint64_t *offset);
int feml_b200_ipc_close(void *base);

/* Expert-sharded mul_mat_id with the combine fused into the GEMM epilogue (no
 * counterpart in the reference): this rank (shard of n_shards == n_peers)
 * computes the slots routed to its experts (expert e on shard e % n_shards,
 * local index e / n_shards) and stores every output column into every rank's
 * output buffer of this step (peer_dst0 / peer_dst1 alternate by *epoch
 * parity as for feml_b200_mul_mat_peer; each buffer holds the full ggml dst,
 * slot (s, t) at + s*dst_nb1 + t*dst_nb2). Slots with an invalid id are zeroed
 * by every rank in its own buffer. The grid's last CTA raises every rank's
 * flag; feml_b200_peer_wait ends the step. Workspace:
 * feml_b200_mul_mat_id_workspace with n_experts = this shard's expert count.
 * Needs the tcgen05 GEMM shapes (quantized, K % 256 == 0, 16-byte aligned
 * rows and activations) and at least one expert per shard. */
int feml_b200_mul_mat_id_peer(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                              int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1, const int32_t *ids,
                              uint64_t ids_nb1, int64_t n_selected, void *const *peer_dst0, void *const *peer_dst1,
                              uint32_t *const *peer_flags, int32_t n_peers, uint64_t dst_nb1, uint64_t dst_nb2,
                              uint32_t *counter, const uint32_t *epoch, int64_t K, int64_t M, int64_t N,
                              void *workspace, uint64_t workspace_bytes, int32_t *status, void *stream);
/* The same step with the combine sent to the token owners (the
 * all-to-all form of the expert-parallel combine; no counterpart in the
 * reference): token t belongs to rank t / owner_tokens (owner_tokens *
 * n_peers >= N), each rank's two buffers hold only its owner_tokens tokens
 * (local token t % owner_tokens at + s*dst_nb1 + (t % owner_tokens)*dst_nb2),
 * and a slot is stored only into its owner's buffer of this step, so a rank
 * sends about 1/n_peers of the slot tensor instead of all of it to every
 * peer. Invalid ids are zeroed by the owner. owner_tokens == 0 is
 * feml_b200_mul_mat_id_peer. */
int feml_b200_mul_mat_id_peer_owned(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2,
                                    int64_t n_experts, int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1,
                                    const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, void *const *peer_dst0,
                                    void *const *peer_dst1, uint32_t *const *peer_flags, int32_t n_peers,
                                    uint64_t dst_nb1, uint64_t dst_nb2, int64_t owner_tokens, uint32_t *counter,
                                    const uint32_t *epoch, int64_t K, int64_t M, int64_t N, void *workspace,
                                    uint64_t workspace_bytes, int32_t *status, void *stream);

/* Enqueue the end of a fused step on this rank: wait (one thread, bounded at
 * about a second) until this rank's flag reaches (*epoch + 1) * n_ranks, then
 * advance *epoch. On timeout bit 0 of *status is set and the stream continues
 * (the context stays usable). */
int feml_b200_peer_wait(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, int32_t *status, void *stream);
/* feml_b200_peer_wait with the bound given: the wait gives up after
 * timeout_us microseconds of the GPU's global timer (1 .. 10,000,000),
 * sets bit 0 (STATUS_TIMEOUT) of *status, leaves *epoch unchanged and lets
 * the stream continue. This is the failure detector of a fused step: a rank
 * that never signals makes its peers' waits run out, not hang. The
 * reference reports failures only as host-side error returns
 * (feml-cpu/tests/cpu_integration.rs:131-144). */
int feml_b200_peer_wait_timeout(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, uint64_t timeout_us,
                                int32_t *status, void *stream);

/* Expert-sharded mul_mat_id (no counterpart in the reference, which has no
 * multi-GPU code): expert e belongs to shard e % n_shards as local expert
 * e / n_shards; w_local holds this shard's local experts (j-th at
 * w_local + j*w_nb2). Writes the dst columns of slots routed to this shard's
 * experts and leaves other shards' columns untouched; invalid ids give zeros
 * and bit 1 of *status as in feml_b200_mul_mat_id. Workspace:
 * feml_b200_mul_mat_id_workspace with n_experts = the local expert count. */
int feml_b200_mul_mat_id_shard(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                               int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1, const int32_t *ids,
                               uint64_t ids_nb1, int64_t n_selected, void *dst, uint64_t dst_nb1, uint64_t dst_nb2,
                               int64_t K, int64_t M, int64_t N, void *workspace, uint64_t workspace_bytes,
                               int32_t *status, void *stream);

/* mul_mat_id routing tables: counts[e], offsets[e] (exclusive prefix sum)
 * and rows[offsets[e] + r] = r-th slot index i = s + t*n_selected routed to
 * e, ascending. Bad ids are skipped and flagged in *status. */
int feml_b200_moe_route(const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, int64_t N, int64_t n_experts,
                        int32_t *counts, int32_t *offsets, int32_t *rows, int32_t *status, void *stream);

/* Per-block int32 sums used by the quantized kernels (for bit-exact
 * checking): out[(m*N + n)*(K/32) + b] = sum over 32-block b of weight
 * integer * activation q8 integer; xq = Q8_0 activations, column n at
 * xq + n*row_size(Q8_0, K). Weight integers: Q8_0 q, Q4_0 nibble-8, Q4_K
 * nibble. */
int feml_b200_block_dots(int32_t wtype, const void *w, uint64_t w_nb1, const void *xq, int64_t K, int64_t M,
                         int64_t N, int32_t *out, void *stream);

/* ---- weight ingestion: host pointers and GGUF files ----------------------- */

/* BackendDevice::buffer_from_host_ptr (feml-core/src/backend.rs:145-153; the
 * reference backends return an error, feml-cuda/src/device.rs:65-72). Wraps
 * `size` bytes of externally owned host memory (an mmap'd model file, for
 * instance) as a new Weights buffer of this backend: the bytes are copied to
 * HBM once, straight from `ptr` (no staging copy), and the handle then
 * behaves like any other buffer (plans address it by handle + offset; the
 * kernels read HBM, not the host link). `max_tensor_size` is the largest
 * tensor the caller will place in the buffer and must not exceed `size`.
 * Blocking; `ptr` need only stay valid for the duration of the call. */
int feml_b200_buffer_from_host_ptr(fb_backend *b, const void *ptr, uint64_t size, uint64_t max_tensor_size,
                                   uint32_t *handle);

/* GGUF reader (the llama.cpp / ggml model container that feml's roadmap names
 * as the source of quantized weights, docs/DESIGN.md:282-286 of the reference: mmap +
 * buffer_from_host_ptr). No counterpart exists in the reference yet; the
 * format follows the public GGUF specification (versions 2 and 3). The file
 * is mapped read-only; every pointer returned stays valid until
 * feml_b200_gguf_close. Malformed files give FB_ERR_INVALID with the
 * offending offset, never an out-of-range read. */
typedef struct fb_gguf fb_gguf;

/* GGUF metadata value types (public specification). */
enum fb_gguf_type {
    FB_GGUF_U8 = 0, FB_GGUF_I8, FB_GGUF_U16, FB_GGUF_I16, FB_GGUF_U32, FB_GGUF_I32, FB_GGUF_F32,
    FB_GGUF_BOOL, FB_GGUF_STRING, FB_GGUF_ARRAY, FB_GGUF_U64, FB_GGUF_I64, FB_GGUF_F64
};

typedef struct {
    char name[256];     /* NUL-terminated */
    int32_t dtype;      /* fb_dtype, or -1 when feml has no counterpart (BF16, IQ types ...) */
    uint32_t ggml_type; /* the file's ggml type id */
    int32_t n_dims;
    int64_t ne[4];      /* ggml order, ne[0] contiguous; unused dimensions are 1 */
    uint64_t offset;    /* byte offset of the data from the start of the file */
    uint64_t nbytes;    /* 0 when the type's block size is unknown */
} fb_gguf_tensor;

int feml_b200_gguf_open(const char *path, fb_gguf **out);
int feml_b200_gguf_close(fb_gguf *g);
int feml_b200_gguf_info(const fb_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *data_offset,
                        int64_t *n_kv, int64_t *n_tensors);
int feml_b200_gguf_tensor(const fb_gguf *g, int64_t index, fb_gguf_tensor *out);
int feml_b200_gguf_find_tensor(const fb_gguf *g, const char *name, int64_t *index);
/* Pointer to the tensor's bytes inside the mapping (nbytes long). */
int feml_b200_gguf_tensor_data(const fb_gguf *g, int64_t index, const void **data);
/* Key `index`: its name (NUL-terminated), value type, array element type
 * (arrays) and count (array elements; string bytes; 1 for scalars). */
int feml_b200_gguf_kv(const fb_gguf *g, int64_t index, const char **key, uint32_t *type, uint32_t *elem_type,
                      uint64_t *count);
int feml_b200_gguf_find_kv(const fb_gguf *g, const char *key, int64_t *index);
/* Scalar values: integers and bools as int64, f32/f64 as double. */
int feml_b200_gguf_kv_int(const fb_gguf *g, int64_t index, int64_t *out);
int feml_b200_gguf_kv_float(const fb_gguf *g, int64_t index, double *out);
/* A string value, or element `elem` of a string array (not NUL-terminated). */
int feml_b200_gguf_kv_str(const fb_gguf *g, int64_t index, int64_t elem, const char **s, uint64_t *len);
/* The first element of a numeric array, inside the mapping (little-endian). */
int feml_b200_gguf_kv_array_data(const fb_gguf *g, int64_t index, const void **data);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* FEML_B200_H */
