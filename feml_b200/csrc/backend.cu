// The B200 backend behind the C ABI (include/feml_b200.h): an implementation
// of feml-core's `Backend` contract (feml-core/src/backend.rs:86-122) for the
// mul_mat / mul_mat_id path.
//
//  - One backend = one device + one non-blocking CUDA stream; all state sits
//    behind a mutex, so it is safe to share between threads (Send + Sync).
//  - Buffers are cudaMalloc'd, zero-initialised and addressed by opaque
//    32-bit handles; every byte range is checked before any copy.
//  - write/read are blocking (feml-cuda/src/backend.rs:96-141); fill and
//    graph_compute are asynchronous until synchronize().
//  - Intermediates (quantized activations, split-K partials, MoE routing
//    tables) live in one device scratch arena. It is sized when a Compute
//    buffer is created and, if a plan's largest node needs more, grown once
//    (synchronizing the device) at that plan's first graph_compute; after
//    that graph_compute allocates nothing.
//  - Kernels record data-dependent failures (bad mul_mat_id ids, a wait that
//    ran out) in a device status word that synchronize() reads and clears.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <unordered_map>
#include <vector>
#include <mutex>
#include <new>

#include "host_common.h"
#include "kernels/common.cuh"
#include "kernels/kernels.h"

using fb::set_error;

namespace fbk {

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cache[dev] = v;
    }
    return cache[dev];
}

}  // namespace fbk

namespace {

constexpr uint64_t kPad = 256;  // slack after every allocation

int cuda_fail(cudaError_t e, const char *what) {
    return set_error(FB_ERR_CUDA, "B200 backend error: %s: %s", what, cudaGetErrorString(e));
}

// mul_mat_id weights: the types the grouped GEMMs tile; mul_mat also takes
// Q5_K and Q6_K (decode GEMV, column groups of up to eight for wider N).
bool is_weight_dtype(int32_t d) { return d == FB_F32 || d == FB_Q8_0 || d == FB_Q4_0 || d == FB_Q4_K; }
bool is_mul_mat_dtype(int32_t d) { return is_weight_dtype(d) || d == FB_Q5_K || d == FB_Q6_K; }

uint64_t align256(uint64_t v) { return (v + 255) / 256 * 256; }

// ---------------------------------------------------------------------------
// mul_mat / mul_mat_id dispatch on device pointers (shared by graph_compute
// and the kernel-level entry points).
// ---------------------------------------------------------------------------
// Shapes for the tcgen05 GEMM, decided from the shape alone so that the
// workspace query and the launch agree (unaligned operands fall back to the
// mma.sync GEMM, which the workspace also covers).
bool tc_shape(int32_t wtype, int64_t K, int64_t M, int64_t N) {
    return !fbk::gemv_supported(wtype, K, N) && fbk::gemm_tc_supported(wtype, K, M, N, nullptr, 0);
}

uint64_t mul_mat_ws(int32_t wtype, int64_t K, int64_t M, int64_t N) {
    if (wtype == FB_F32) return 0;
    if (fbk::gemv_supported(wtype, K, N) && fbk::gemv_fused_ok(K, N)) return 0;
    // planar activations + split-K partials for the mma.sync GEMM; the
    // tcgen05 path needs the hi/lo activations instead
    const uint64_t planar = fbk::q8_planar_bytes(K, N) + fbk::gemm_q_split_bytes(K, M, N);
    return tc_shape(wtype, K, M, N) ? std::max<uint64_t>(planar, fbk::xq16_bytes(wtype, K, N, M, false)) : planar;
}

// Kernel launches one do_mul_mat of this shape enqueues (16-byte aligned
// operands), from the same dispatch decisions do_mul_mat takes.
int mul_mat_launches(int32_t wtype, int64_t K, int64_t M, int64_t N) {
    if (M <= 0 || N <= 0) return 0;
    if (wtype == FB_F32) return 1;
    if (mul_mat_ws(wtype, K, M, N) == 0) return 1;  // fused decode GEMV
    if (tc_shape(wtype, K, M, N))
        return fbk::gemm_tc_splits(wtype, K, M, N) > 1 || fbk::gemm_tc_tail(wtype, K, M, N, nullptr) ? 3 : 2;
    if (fbk::gemv_supported(wtype, K, N)) return 2;
    const int64_t rb = fb::row_size(wtype, K);
    if (rb > 0 && fbk::gemm_q_supported(wtype, K, nullptr, (uint64_t)rb))
        return fbk::gemm_q_splits(K, M, N) > 1 ? 3 : 2;
    return 1 + (int)((N + fbk::gemv_max_cols() - 1) / fbk::gemv_max_cols());
}

// norm_eps non-null: x is rms-normalized (that eps) inside the decode GEMV
// (graph_compute passes it only for shapes where that path runs).
// epi non-null: the bias / SiLU epilogue of a fused mul_mat -> add -> silu
// chain: inside the decode GEMV and the tcgen05 GEMM, or as one pass over y
// after the other kernels (same arithmetic, same bits).
int do_mul_mat(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y, uint64_t y_nb1,
               int64_t K, int64_t M, int64_t N, void *ws, uint64_t ws_bytes, int32_t *status, cudaStream_t s,
               const float *norm_eps = nullptr, const fbk::EpiAct *epi = nullptr) {
    if (K < 0 || M < 0 || N < 0) return set_error(FB_ERR_INVALID, "mul_mat: negative dimension");
    if (M == 0 || N == 0) return FB_OK;
    if (!w || !x || !y) return set_error(FB_ERR_INVALID, "mul_mat: null operand");
    if (!is_mul_mat_dtype(wtype)) return set_error(FB_ERR_UNSUPPORTED, "mul_mat: weight dtype %d not supported", wtype);
    const fb::DTypeTraits *t = fb::dtype_traits(wtype);
    if (K % t->block_size) return set_error(FB_ERR_SHAPE, "mul_mat: K %ld not a multiple of %ld", (long)K, (long)t->block_size);
    const bool act = fbk::epi_active(epi);
    // kernels without a fused epilogue: one bias / SiLU pass over y afterwards
    auto then_act = [&](int rc) { return rc || !act ? rc : fbk::launch_bias_act(y, y_nb1, M, N, *epi, s); };
    if (wtype == FB_F32) return then_act(fbk::launch_gemm_f32(w, w_nb1, x, x_nb1, y, y_nb1, K, M, N, status, s));
    if (K == 0) return set_error(FB_ERR_SHAPE, "mul_mat: K == 0");

    const uint64_t need = mul_mat_ws(wtype, K, M, N);
    if (need > ws_bytes)
        return set_error(FB_ERR_INVALID, "mul_mat: workspace of %lu bytes needed, %lu given", (unsigned long)need,
                         (unsigned long)ws_bytes);
    if (need == 0)
        return fbk::launch_gemv(wtype, w, w_nb1, x, x_nb1, y, y_nb1, K, M, N, nullptr, status, s, true, nullptr,
                                norm_eps, epi);
    if (norm_eps) return set_error(FB_ERR_UNSUPPORTED, "mul_mat: fused rms_norm needs the decode GEMV");
    if (tc_shape(wtype, K, M, N) && fbk::gemm_tc_supported(wtype, K, M, N, w, w_nb1) &&
        ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15) == 0) {
        const fbk::XQ16 xa = fbk::xq16_carve(wtype, ws, K, N);
        int rc = fbk::launch_quantize_q8_f16(x, x_nb1, K, N, xa, nullptr, s, wtype);
        if (rc) return rc;
        return fbk::launch_gemm_tc(wtype, w, w_nb1, xa, K, M, N, y, y_nb1, nullptr, status, s, nullptr, epi);
    }

    const fbk::Q8Planar xq = fbk::q8_planar_carve(ws, K, N);
    int rc = fbk::launch_quantize_q8_planar(x, x_nb1, K, N, xq, s);
    if (rc) return rc;
    if (fbk::gemv_supported(wtype, K, N))
        return fbk::launch_gemv(wtype, w, w_nb1, x, x_nb1, y, y_nb1, K, M, N, &xq, status, s, true, nullptr, nullptr,
                                epi);
    if (fbk::gemm_q_supported(wtype, K, w, w_nb1))
        return then_act(fbk::launch_gemm_q(wtype, w, w_nb1, xq, K, M, N, y, y_nb1, nullptr, s,
                                           static_cast<uint8_t *>(ws) + fbk::q8_planar_bytes(K, N)));
    // Shapes the GEMM cannot tile (K % 256 != 0, unaligned rows): the GEMV on
    // groups of up to gemv_max_cols() columns of the already-quantized
    // activations.
    const int64_t nblk = K / 32, ncol = fbk::gemv_max_cols();
    for (int64_t n0 = 0; n0 < N; n0 += ncol) {
        const int64_t nc = std::min<int64_t>(ncol, N - n0);
        fbk::Q8Planar sub{xq.qs + n0 * K, xq.d + n0 * nblk, xq.sum + n0 * nblk};
        rc = fbk::launch_gemv(wtype, w, w_nb1, x, x_nb1, static_cast<uint8_t *>(y) + n0 * y_nb1, y_nb1, K, M, nc,
                              &sub, status, s, false, nullptr, nullptr, epi);
        if (rc) return rc;
    }
    return FB_OK;
}

struct IdWorkspace {
    int32_t *counts, *offsets, *tile_start, *rows;
    void *xq;
    uint64_t total;
};

// mul_mat_id shapes for the tcgen05 GEMM (shape-only, as for mul_mat).
bool id_tc_shape(int32_t wtype, int64_t K, int64_t N, int64_t n_sel) {
    return fbk::gemm_tc_supported(wtype, K, 1, N * n_sel, nullptr, 0);
}

IdWorkspace id_ws_layout(void *base, int32_t wtype, int64_t K, int64_t N, int64_t n_sel, int64_t E) {
    IdWorkspace L{};
    uint8_t *p = static_cast<uint8_t *>(base);
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        uint8_t *r = p ? p + off : nullptr;
        off += align256(bytes);
        return r;
    };
    L.counts = reinterpret_cast<int32_t *>(take(4 * E));
    L.offsets = reinterpret_cast<int32_t *>(take(4 * E));
    L.tile_start = reinterpret_cast<int32_t *>(take(4 * (E + 1)));
    L.rows = reinterpret_cast<int32_t *>(take(4 * n_sel * N));
    uint64_t xq_bytes = fbk::q8_planar_bytes(K, N);
    if (id_tc_shape(wtype, K, N, n_sel)) xq_bytes = std::max<uint64_t>(xq_bytes, fbk::xq16_bytes(wtype, K, N * n_sel, 0, true));
    L.xq = wtype == FB_F32 ? nullptr : take(xq_bytes);
    L.total = off;
    return L;
}

// Expert-sharded form: `w` holds this shard's experts (local expert j = global
// expert shard + j*n_shards, j-th at w + j*w_nb2); slots routed to other
// shards are left untouched. shard = 0, n_shards = 1 is plain mul_mat_id.
int do_mul_mat_id(int32_t wtype, const void *w, uint64_t w_nb1, uint64_t w_nb2, int64_t E, int64_t shard,
                  int64_t n_shards, const void *x, uint64_t x_nb1, const int32_t *ids, uint64_t ids_nb1,
                  int64_t n_sel, void *dst, uint64_t dst_nb1, uint64_t dst_nb2, int64_t K, int64_t M, int64_t N,
                  void *ws, uint64_t ws_bytes, int32_t *status, cudaStream_t s) {
    if (K < 0 || M < 0 || N < 0 || n_sel < 1 || E < 1) return set_error(FB_ERR_INVALID, "mul_mat_id: bad dimensions");
    if (n_shards < 1 || shard < 0 || shard >= n_shards) return set_error(FB_ERR_INVALID, "mul_mat_id: bad shard");
    if (M == 0 || N == 0) return FB_OK;
    const int64_t n_local = fbk::local_experts(E, shard, n_shards);
    // a shard that owns no expert still routes (invalid ids are zeroed and reported)
    if ((!w && n_local > 0) || !x || !ids || !dst) return set_error(FB_ERR_INVALID, "mul_mat_id: null operand");
    if (!is_weight_dtype(wtype)) return set_error(FB_ERR_UNSUPPORTED, "mul_mat_id: weight dtype %d not supported", wtype);
    const fb::DTypeTraits *t = fb::dtype_traits(wtype);
    if (K % t->block_size) return set_error(FB_ERR_SHAPE, "mul_mat_id: K not a block multiple");
    const IdWorkspace need = id_ws_layout(nullptr, wtype, K, N, n_sel, n_local);
    if (need.total > ws_bytes)
        return set_error(FB_ERR_INVALID, "mul_mat_id: workspace of %lu bytes needed, %lu given",
                         (unsigned long)need.total, (unsigned long)ws_bytes);
    const IdWorkspace L = id_ws_layout(ws, wtype, K, N, n_sel, n_local);
    const bool use_tc = id_tc_shape(wtype, K, N, n_sel) && n_local > 0 &&
                        fbk::gemm_tc_supported(wtype, K, M, N * n_sel, w, w_nb1) && (w_nb2 & 15) == 0 &&
                        ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15) == 0;
    const int block_n = wtype == FB_F32 ? fbk::gemm_f32_block_n()
                        : use_tc        ? fbk::gemm_tc_block_n(wtype, K)
                                        : fbk::gemm_q_block_n();
    if (wtype != FB_F32 && !use_tc && !fbk::gemm_q_supported(wtype, K, w, w_nb1))
        return set_error(FB_ERR_UNSUPPORTED, "mul_mat_id: quantized experts need K %% 256 == 0 and 16-byte aligned rows");
    int rc = fbk::launch_moe_route(ids, ids_nb1, n_sel, N, E, shard, n_shards, L.counts, L.offsets, L.rows,
                                   L.tile_start, block_n, status, dst, dst_nb1, dst_nb2, M, s);
    if (rc) return rc;
    fbk::GroupMap g{};
    g.counts = L.counts;
    g.offsets = L.offsets;
    g.rows = L.rows;
    g.tile_start = L.tile_start;
    g.n_groups = (int32_t)n_local;
    g.n_selected = (int32_t)n_sel;
    g.w_group_stride = w_nb2;
    g.dst_nb1 = dst_nb1;
    g.dst_nb2 = dst_nb2;
    g.max_tiles = (int32_t)((n_sel * N + block_n - 1) / block_n + n_local);
    if (n_local == 0) return FB_OK;
    if (wtype == FB_F32) return fbk::launch_gemm_f32_grouped(w, w_nb1, x, x_nb1, K, M, dst, g, s);
    if (use_tc) {
        const fbk::XQ16 xa = fbk::xq16_carve(wtype, L.xq, K, N * n_sel);
        rc = fbk::launch_quantize_q8_f16(x, x_nb1, K, N, xa, &g, s, wtype);
        if (rc) return rc;
        return fbk::launch_gemm_tc(wtype, w, w_nb1, xa, K, M, N, dst, 0, &g, status, s);
    }
    const fbk::Q8Planar xq = fbk::q8_planar_carve(L.xq, K, N);
    rc = fbk::launch_quantize_q8_planar(x, x_nb1, K, N, xq, s);
    if (rc) return rc;
    return fbk::launch_gemm_q(wtype, w, w_nb1, xq, K, M, 0, dst, 0, &g, s);
}

}  // namespace

// ---------------------------------------------------------------------------
// Backend object
// ---------------------------------------------------------------------------
struct Buffer {
    uint8_t *ptr;
    uint64_t size;
    int32_t usage;
};

struct fb_backend {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::map<uint32_t, Buffer> buffers;
    uint32_t next_handle = 1;
    void *scratch = nullptr;
    uint64_t scratch_bytes = 0;
    int32_t *status_dev = nullptr;
    int32_t *status_host = nullptr;  // pinned
    uint64_t device_allocs = 0;      // cudaMalloc calls made for buffers and scratch
    uint8_t *stage = nullptr;        // pinned staging area of small writes
    cudaEvent_t stage_free = nullptr;  // recorded after the last staged copy
    // Executable CUDA graphs of plans already run, keyed by a hash of every
    // plan field the launches depend on; `key` holds those fields for an
    // exact comparison; exec == nullptr marks a plan whose capture failed
    // (it runs node by node).
    struct PlanGraph {
        std::vector<uint64_t> key;
        cudaGraphExec_t exec = nullptr;
    };
    std::unordered_map<uint64_t, PlanGraph> graphs;
    bool use_graphs = true;
};

// Writes up to this size are copied into the pinned staging area and sent
// to the device by an asynchronous copy on the backend stream, so write()
// returns without a stream synchronize (the caller's bytes are already
// copied, and every later use of the buffer is ordered after the copy on the
// same stream). Larger writes copy directly and synchronize.
constexpr uint64_t kStageBytes = 1u << 20;

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int lookup(fb_backend *b, uint32_t h, const char *op, Buffer **out) {
    auto it = b->buffers.find(h);
    if (it == b->buffers.end()) return set_error(FB_ERR_INVALID, "%s: unknown buffer buf#%u", op, h);
    *out = &it->second;
    return FB_OK;
}

int check_range(const Buffer &buf, uint32_t h, uint64_t off, uint64_t n, const char *op) {
    if (off > buf.size || n > buf.size - off)
        return set_error(FB_ERR_INVALID, "%s: buf#%u overflow: offset %lu + %lu > buffer %lu", op, h,
                         (unsigned long)off, (unsigned long)n, (unsigned long)buf.size);
    return FB_OK;
}

// Drop every cached plan graph: they hold buffer and scratch addresses.
// Callers have synchronized the stream, so none is executing.
void clear_plan_graphs(fb_backend *b) {
    for (auto &kv : b->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    b->graphs.clear();
}

int grow_scratch(fb_backend *b, uint64_t bytes) {
    if (bytes <= b->scratch_bytes) return FB_OK;
    bytes = align256(bytes);
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return cuda_fail(e, "scratch sync");
    clear_plan_graphs(b);
    if (b->scratch) cudaFree(b->scratch);
    b->scratch = nullptr;
    b->scratch_bytes = 0;
    e = cudaMalloc(&b->scratch, bytes);
    b->device_allocs++;
    if (e != cudaSuccess) {
        b->scratch = nullptr;
        return cuda_fail(e, "scratch alloc");
    }
    b->scratch_bytes = bytes;
    return FB_OK;
}

// A plan tensor resolved to device memory.
struct DevTensor {
    const fb_plan_tensor *t;
    uint8_t *ptr;
    uint32_t handle;
    uint64_t nbytes;
};

int resolve(fb_backend *b, const fb_plan *plan, int64_t idx, DevTensor *out) {
    if (idx < 0 || idx >= plan->n_tensors) return set_error(FB_ERR_INVALID, "graph_compute: tensor index %ld out of range", (long)idx);
    const fb_plan_tensor &t = plan->tensors[idx];
    if (t.buffer < 0 || t.buffer >= plan->n_buffers)
        return set_error(FB_ERR_INVALID, "graph_compute: tensor %u has no buffer", t.id);
    const uint32_t h = plan->buffers[t.buffer].handle;
    Buffer *buf;
    int rc = lookup(b, h, "graph_compute", &buf);
    if (rc) return rc;
    uint64_t nb = 0;
    rc = fb_layout_nbytes(t.dtype, t.ne, t.nb, &nb);
    if (rc) return rc;
    rc = check_range(*buf, h, t.offset, nb, "graph_compute");
    if (rc) return rc;
    out->t = &t;
    out->ptr = buf->ptr + t.offset;
    out->handle = h;
    out->nbytes = nb;
    return FB_OK;
}

bool overlap(const DevTensor &a, const DevTensor &c) {
    if (a.handle != c.handle) return false;
    const uint64_t ao = a.t->offset, co = c.t->offset;
    return ao < co + c.nbytes && co < ao + a.nbytes;
}

// ---- rms_norm and its fusion into mul_mat ----------------------------------
float rms_eps(const fb_plan_tensor &t) {
    float eps;
    std::memcpy(&eps, &t.op_params[0], 4);
    return eps;
}

bool ranges_overlap(const fb_plan *plan, const fb_plan_tensor &a, const fb_plan_tensor &c) {
    if (a.buffer != c.buffer || a.buffer < 0) return false;
    uint64_t an = 0, cn = 0;
    if (fb_layout_nbytes(a.dtype, a.ne, a.nb, &an) || fb_layout_nbytes(c.dtype, c.ne, c.nb, &cn)) return true;
    return a.offset < c.offset + cn && c.offset < a.offset + an;
}

// An rms_norm node runs inside the decode GEMV of its consumers instead of
// on its own when nothing else can see its output: it is not a graph
// output, every reader is a mul_mat taking it as activations whose shape
// runs on the in-kernel-quantizing GEMV (quantized weights, N*K <= 16384,
// K >= 512), those readers follow it directly in the node order, and none
// of their outputs overlaps the normalized tensor's source (the planner may
// reuse that memory once the rms_norm would have consumed it).
bool rms_fused(const fb_plan *plan, int64_t ri) {
    if (ri < 0 || ri >= plan->n_tensors) return false;
    const fb_plan_tensor &r = plan->tensors[ri];
    if (r.op != FB_OP_RMS_NORM || (r.flags & FB_FLAG_OUTPUT) || r.n_srcs != 1 || r.dtype != FB_F32) return false;
    if (r.srcs[0] < 0 || r.srcs[0] >= plan->n_tensors) return false;
    const fb_plan_tensor &x = plan->tensors[r.srcs[0]];
    if (x.dtype != FB_F32 || x.nb[0] != 4 || x.ne[2] != 1 || x.ne[3] != 1) return false;
    const int64_t K = x.ne[0], N = x.ne[1];
    if (K < 512 || N < 1 || !fbk::gemv_fused_ok(K, N)) return false;
    int64_t consumers = 0;
    for (int64_t i = 0; i < plan->n_tensors; i++) {
        const fb_plan_tensor &t = plan->tensors[i];
        for (int k = 0; k < t.n_srcs && k < FB_MAX_SRC; k++) {
            if (t.srcs[k] != ri) continue;
            if (t.op != FB_OP_MUL_MAT || k != 1 || t.srcs[0] < 0 || t.srcs[0] >= plan->n_tensors) return false;
            const fb_plan_tensor &w = plan->tensors[t.srcs[0]];
            if (w.dtype == FB_F32 || !fbk::gemv_supported(w.dtype, K, N) || ranges_overlap(plan, x, t)) return false;
            consumers++;
        }
    }
    if (consumers == 0) return false;
    int64_t pos = -1;
    for (int64_t i = 0; i < plan->n_nodes; i++)
        if (plan->nodes[i] == ri) pos = i;
    if (pos < 0) return false;
    int64_t seen = 0;
    for (int64_t i = pos + 1; i < plan->n_nodes && seen < consumers; i++) {
        const int64_t ti = plan->nodes[i];
        if (ti < 0 || ti >= plan->n_tensors) return false;
        const fb_plan_tensor &t = plan->tensors[ti];
        if (t.op != FB_OP_MUL_MAT || t.n_srcs < 2 || t.srcs[1] != ri) return false;
        seen++;
    }
    return seen == consumers;
}

int compute_rms_norm(fb_backend *b, const fb_plan *plan, const fb_plan_tensor &node) {
    if (node.n_srcs != 1) return set_error(FB_ERR_INVALID, "rms_norm: expected 1 source");
    DevTensor X, Y;
    int rc;
    if ((rc = resolve(b, plan, node.srcs[0], &X)) || (rc = resolve(b, plan, &node - plan->tensors, &Y))) return rc;
    const fb_plan_tensor &x = *X.t, &y = *Y.t;
    if (x.dtype != FB_F32 || y.dtype != FB_F32) return set_error(FB_ERR_UNSUPPORTED, "B200: rms_norm needs f32");
    for (int d = 0; d < 4; d++)
        if (x.ne[d] != y.ne[d]) return set_error(FB_ERR_SHAPE, "shape error: rms_norm: dst shape differs from src");
    // in place (y == x) is allowed (op.rs:98-110); any other overlap is not
    if (overlap(X, Y) && X.ptr != Y.ptr) return set_error(FB_ERR_INVALID, "B200: rms_norm dst partly aliases src");
    return fbk::launch_rms_norm(X.ptr, x.nb, Y.ptr, y.nb, y.ne, rms_eps(node), b->stream);
}

// ---- mul_mat -> add(bias) -> silu fusion --------------------------------
// A mul_mat whose output is read only by a bias add (the other operand a
// vector of M floats broadcast over the N columns) and/or a SiLU, each
// intermediate read by nothing else, not a graph output and computed by the
// very next node, runs as one kernel: the chain's last tensor is written by
// the mul_mat's epilogue and the add / silu nodes are skipped (the
// compile-time fusion of the reference's roadmap, docs/DESIGN.md:251).
struct ActChain {
    int64_t add = -1, silu = -1;  // fused nodes (tensor indices)
    int64_t bias = -1;            // the bias vector
    int64_t out = -1;             // the tensor the mul_mat kernel writes
};

// The only tensor that reads tensor `ti` (-1 when none or several do).
int64_t sole_reader(const fb_plan *plan, int64_t ti) {
    int64_t r = -1, n = 0;
    for (int64_t i = 0; i < plan->n_tensors; i++) {
        const fb_plan_tensor &t = plan->tensors[i];
        for (int k = 0; k < t.n_srcs && k < FB_MAX_SRC; k++)
            if (t.srcs[k] == ti) {
                r = i;
                n++;
            }
    }
    return n == 1 ? r : -1;
}

bool f32_2d(const fb_plan_tensor &t, int64_t M, int64_t N) {
    return t.dtype == FB_F32 && t.ne[0] == M && t.ne[1] == N && t.ne[2] == 1 && t.ne[3] == 1 && t.nb[0] == 4;
}

// The chain starting at the mul_mat at node position `pos`, or none.
ActChain act_chain(const fb_plan *plan, int64_t pos) {
    ActChain c;
    const int64_t mi = plan->nodes[pos];
    const fb_plan_tensor &mm = plan->tensors[mi];
    const int64_t M = mm.ne[0], N = mm.ne[1];
    if (mm.op != FB_OP_MUL_MAT || (mm.flags & FB_FLAG_OUTPUT) || !f32_2d(mm, M, N)) return c;
    auto next_is = [&](int64_t p, int64_t t) { return p < plan->n_nodes && plan->nodes[p] == t; };
    const int64_t r1 = sole_reader(plan, mi);
    if (r1 < 0 || !next_is(pos + 1, r1)) return c;
    const fb_plan_tensor &t1 = plan->tensors[r1];
    ActChain found;
    if (t1.op == FB_OP_ADD && t1.n_srcs == 2 && f32_2d(t1, M, N)) {
        const int64_t bi = t1.srcs[0] == mi ? t1.srcs[1] : t1.srcs[0];
        if (bi < 0 || bi >= plan->n_tensors || bi == mi || (t1.srcs[0] != mi && t1.srcs[1] != mi)) return c;
        const fb_plan_tensor &bt = plan->tensors[bi];
        if (bt.dtype != FB_F32 || bt.ne[0] != M || bt.ne[1] != 1 || bt.ne[2] != 1 || bt.ne[3] != 1 || bt.nb[0] != 4)
            return c;
        found.add = r1;
        found.bias = bi;
        found.out = r1;
        const int64_t r2 = (t1.flags & FB_FLAG_OUTPUT) ? -1 : sole_reader(plan, r1);
        if (r2 >= 0 && next_is(pos + 2, r2)) {
            const fb_plan_tensor &t2 = plan->tensors[r2];
            if (t2.op == FB_OP_SILU && t2.n_srcs == 1 && f32_2d(t2, M, N)) {
                found.silu = r2;
                found.out = r2;
            }
        }
    } else if (t1.op == FB_OP_SILU && t1.n_srcs == 1 && f32_2d(t1, M, N)) {
        found.silu = r1;
        found.out = r1;
    } else {
        return c;
    }
    // the kernel writes `out` while reading the weights, the activations and
    // the bias: none of them may share its bytes (the mul_mat's own output
    // and the add's are never materialized, so `out` may reuse them)
    const fb_plan_tensor &o = plan->tensors[found.out];
    const int64_t reads[3] = {mm.srcs[0], mm.srcs[1], found.bias};
    for (int64_t ri : reads)
        if (ri >= 0 && ri < plan->n_tensors && ranges_overlap(plan, plan->tensors[ri], o)) return c;
    return found;
}

int compute_mul_mat(fb_backend *b, const fb_plan *plan, const fb_plan_tensor &node, const ActChain *chain = nullptr) {
    if (node.n_srcs != 2) return set_error(FB_ERR_INVALID, "mul_mat: expected 2 sources");
    DevTensor A, B, C;
    int rc;
    // activations from a fused rms_norm: read its source and normalize in the GEMV
    const int64_t act = node.srcs[1];
    const bool fused_norm = rms_fused(plan, act);
    float eps = 0.0f;
    if (fused_norm) eps = rms_eps(plan->tensors[act]);
    if ((rc = resolve(b, plan, node.srcs[0], &A)) ||
        (rc = resolve(b, plan, fused_norm ? plan->tensors[act].srcs[0] : act, &B)))
        return rc;
    if ((rc = resolve(b, plan, chain ? chain->out : &node - plan->tensors, &C))) return rc;
    fbk::EpiAct epi{nullptr, 0};
    if (chain) {
        if (chain->bias >= 0) {
            DevTensor Bias;
            if ((rc = resolve(b, plan, chain->bias, &Bias))) return rc;
            if (overlap(Bias, C)) return set_error(FB_ERR_INVALID, "B200: fused mul_mat dst aliases the bias");
            epi.bias = reinterpret_cast<const float *>(Bias.ptr);
        }
        epi.silu = chain->silu >= 0 ? 1 : 0;
    }
    if (overlap(A, C) || overlap(B, C)) return set_error(FB_ERR_INVALID, "B200: mul_mat dst aliases a source");
    const fb_plan_tensor &a = *A.t, &x = *B.t, &y = *C.t;
    if (!is_mul_mat_dtype(a.dtype) || x.dtype != FB_F32 || y.dtype != FB_F32)
        return set_error(FB_ERR_UNSUPPORTED, "B200: mul_mat dtypes not supported");
    const int64_t K = a.ne[0], M = a.ne[1], N = x.ne[1];
    if (x.ne[0] != K || y.ne[0] != M || y.ne[1] != N)
        return set_error(FB_ERR_SHAPE, "shape error: mul_mat: dst %ldx%ld but expected %ldx%ld", (long)y.ne[0],
                         (long)y.ne[1], (long)M, (long)N);
    if (a.ne[2] != 1 || a.ne[3] != 1 || x.ne[2] != 1 || x.ne[3] != 1 || y.ne[2] != 1 || y.ne[3] != 1)
        return set_error(FB_ERR_SHAPE, "shape error: mul_mat: rank > 2 not supported yet");
    if (a.nb[0] != (uint64_t)fb::dtype_traits(a.dtype)->type_size || x.nb[0] != 4 || y.nb[0] != 4)
        return set_error(FB_ERR_UNSUPPORTED, "B200: mul_mat needs contiguous rows");
    return do_mul_mat(a.dtype, A.ptr, a.nb[1], B.ptr, x.nb[1], C.ptr, y.nb[1], K, M, N, b->scratch, b->scratch_bytes,
                      b->status_dev, b->stream, fused_norm ? &eps : nullptr, chain ? &epi : nullptr);
}

// Standalone add (feml-cpu/src/ops/elementwise.rs semantics: ggml
// broadcasting; dst may alias a source exactly, any partial overlap is
// rejected, as in feml-cpu/src/backend.rs:193-204).
int compute_add(fb_backend *b, const fb_plan *plan, const fb_plan_tensor &node) {
    if (node.n_srcs != 2) return set_error(FB_ERR_INVALID, "add: expected 2 sources");
    DevTensor X, Y, Z;
    int rc;
    if ((rc = resolve(b, plan, node.srcs[0], &X)) || (rc = resolve(b, plan, node.srcs[1], &Y)) ||
        (rc = resolve(b, plan, &node - plan->tensors, &Z)))
        return rc;
    if (X.t->dtype != FB_F32 || Y.t->dtype != FB_F32 || Z.t->dtype != FB_F32)
        return set_error(FB_ERR_UNSUPPORTED, "B200: add needs f32");
    for (const DevTensor *S : {&X, &Y})
        if (overlap(*S, Z) && (S->ptr != Z.ptr || S->nbytes != Z.nbytes))
            return set_error(FB_ERR_INVALID, "B200: partial-overlap alias not supported");
    return fbk::launch_add_f32(X.ptr, X.t->ne, X.t->nb, Y.ptr, Y.t->ne, Y.t->nb, Z.ptr, Z.t->ne, Z.t->nb, b->stream);
}

int compute_silu(fb_backend *b, const fb_plan *plan, const fb_plan_tensor &node) {
    if (node.n_srcs != 1) return set_error(FB_ERR_INVALID, "silu: expected 1 source");
    DevTensor X, Y;
    int rc;
    if ((rc = resolve(b, plan, node.srcs[0], &X)) || (rc = resolve(b, plan, &node - plan->tensors, &Y))) return rc;
    if (X.t->dtype != FB_F32 || Y.t->dtype != FB_F32) return set_error(FB_ERR_UNSUPPORTED, "B200: silu needs f32");
    for (int d = 0; d < 4; d++)
        if (X.t->ne[d] != Y.t->ne[d]) return set_error(FB_ERR_SHAPE, "shape error: silu: dst shape differs from src");
    if (overlap(X, Y) && X.ptr != Y.ptr) return set_error(FB_ERR_INVALID, "B200: silu dst partly aliases src");
    return fbk::launch_silu_f32(X.ptr, X.t->nb, Y.ptr, Y.t->nb, Y.t->ne, b->stream);
}

int compute_mul_mat_id(fb_backend *b, const fb_plan *plan, const fb_plan_tensor &node) {
    if (node.n_srcs != 3) return set_error(FB_ERR_INVALID, "mul_mat_id: expected 3 sources");
    DevTensor W, X, I, D;
    int rc;
    if ((rc = resolve(b, plan, node.srcs[0], &W)) || (rc = resolve(b, plan, node.srcs[1], &X)) ||
        (rc = resolve(b, plan, node.srcs[2], &I)))
        return rc;
    if ((rc = resolve(b, plan, &node - plan->tensors, &D))) return rc;
    if (overlap(W, D) || overlap(X, D) || overlap(I, D))
        return set_error(FB_ERR_INVALID, "B200: mul_mat_id dst aliases a source");
    const fb_plan_tensor &w = *W.t, &x = *X.t, &ids = *I.t, &d = *D.t;
    if (!is_weight_dtype(w.dtype) || x.dtype != FB_F32 || ids.dtype != FB_I32 || d.dtype != FB_F32)
        return set_error(FB_ERR_UNSUPPORTED, "B200: mul_mat_id dtypes not supported");
    const int64_t K = w.ne[0], M = w.ne[1], E = w.ne[2], N = x.ne[1], n_sel = ids.ne[0];
    if (x.ne[0] != K || ids.ne[1] != N || d.ne[0] != M || d.ne[1] != n_sel || d.ne[2] != N || w.ne[3] != 1)
        return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: inconsistent shapes");
    if (w.nb[0] != (uint64_t)fb::dtype_traits(w.dtype)->type_size || x.nb[0] != 4 || ids.nb[0] != 4 || d.nb[0] != 4)
        return set_error(FB_ERR_UNSUPPORTED, "B200: mul_mat_id needs contiguous rows");
    return do_mul_mat_id(w.dtype, W.ptr, w.nb[1], w.nb[2], E, 0, 1, X.ptr, x.nb[1], reinterpret_cast<int32_t *>(I.ptr),
                         ids.nb[1], n_sel, D.ptr, d.nb[1], d.nb[2], K, M, N, b->scratch, b->scratch_bytes,
                         b->status_dev, b->stream);
}

// vtable adapters
const char *vt_name(void *) { return "B200"; }
int vt_create(void *c, uint64_t size, int32_t usage, uint32_t *h) {
    return feml_b200_create_buffer(static_cast<fb_backend *>(c), size, usage, h);
}
int vt_release(void *c, uint32_t h) { return feml_b200_release_buffer(static_cast<fb_backend *>(c), h); }
int vt_write(void *c, uint32_t h, uint64_t o, const void *s, uint64_t n) {
    return feml_b200_write(static_cast<fb_backend *>(c), h, o, s, n);
}
int vt_read(void *c, uint32_t h, uint64_t o, void *d, uint64_t n) {
    return feml_b200_read(static_cast<fb_backend *>(c), h, o, d, n);
}
int vt_fill(void *c, uint32_t h, uint64_t o, uint8_t v, uint64_t n) {
    return feml_b200_fill(static_cast<fb_backend *>(c), h, o, v, n);
}
int vt_sync(void *c) { return feml_b200_synchronize(static_cast<fb_backend *>(c)); }
int vt_compute(void *c, const fb_plan *p) { return feml_b200_graph_compute(static_cast<fb_backend *>(c), p); }
int vt_supports(void *c, int32_t op, const int32_t *d, int32_t n) {
    return feml_b200_supports_op(static_cast<fb_backend *>(c), op, d, n);
}
int vt_prepare(void *c, const fb_plan *p) { return feml_b200_prepare_plan(static_cast<fb_backend *>(c), p); }

bool is_sm100(int dev) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return false;
    return prop.major == 10 && prop.minor == 0;
}

}  // namespace

extern "C" {

int feml_b200_device_count(int32_t *count) {
    if (!count) return set_error(FB_ERR_INVALID, "device_count: null out");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();  // no driver / no device: an empty registrar, not an error
        n = 0;
    }
    int c = 0;
    for (int d = 0; d < n; d++)
        if (is_sm100(d)) c++;
    *count = c;
    return FB_OK;
}

int feml_b200_registrar_score(uint32_t *score) {
    int32_t n = 0;
    feml_b200_device_count(&n);
    if (score) *score = n > 0 ? 2000u : 0u;
    return FB_OK;
}

int feml_b200_device_info(int32_t device, fb_device_info *info) {
    if (!info) return set_error(FB_ERR_INVALID, "device_info: null out");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return set_error(FB_ERR_NO_DEVICE, "B200: device %d not found", device);
    }
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "device properties");
    memset(info, 0, sizeof(*info));
    snprintf(info->name, sizeof(info->name), "%s", prop.name);
    {
        DeviceGuard g(device);
        size_t fr = 0, tot = 0;
        if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) {
            info->memory_free = fr;
            info->memory_total = tot;
        }
    }
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    info->sm_count = prop.multiProcessorCount;
    info->device_type = 1;
    info->async_compute = 1;
    info->host_buffer = 1;  // buffer_from_host_ptr (copied to HBM)
    info->events = 1;
    return FB_OK;
}

int feml_b200_open(int32_t device, fb_backend **out) {
    if (!out) return set_error(FB_ERR_INVALID, "open: null out");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return set_error(FB_ERR_NO_DEVICE, "B200: device %d not found", device);
    }
    if (!is_sm100(device)) return set_error(FB_ERR_NO_DEVICE, "B200: device %d is not an sm_100 GPU", device);
    fb_backend *b = new (std::nothrow) fb_backend();
    if (!b) return set_error(FB_ERR_INVALID, "open: out of host memory");
    b->device = device;
    DeviceGuard g(device);
    cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&b->status_dev, 256);
    if (e == cudaSuccess) e = cudaMemset(b->status_dev, 0, 256);
    if (e == cudaSuccess) e = cudaMallocHost(&b->status_host, 256);
    if (e == cudaSuccess) e = cudaMallocHost(&b->stage, kStageBytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b->stage_free, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(b->stage_free, b->stream);
    if (e != cudaSuccess) {
        int rc = cuda_fail(e, "open");
        feml_b200_close(b);
        return rc;
    }
    fbk::sm_count();
    *out = b;
    return FB_OK;
}

int feml_b200_close(fb_backend *b) {
    if (!b) return FB_OK;
    {
        DeviceGuard g(b->device);
        if (b->stream) cudaStreamSynchronize(b->stream);
        clear_plan_graphs(b);
        for (auto &kv : b->buffers) cudaFree(kv.second.ptr);
        if (b->scratch) cudaFree(b->scratch);
        if (b->status_dev) cudaFree(b->status_dev);
        if (b->status_host) cudaFreeHost(b->status_host);
        if (b->stage) cudaFreeHost(b->stage);
        if (b->stage_free) cudaEventDestroy(b->stage_free);
        if (b->stream) cudaStreamDestroy(b->stream);
    }
    delete b;
    return FB_OK;
}

const char *feml_b200_name(fb_backend *) { return "B200"; }

int feml_b200_create_buffer(fb_backend *b, uint64_t size, int32_t usage, uint32_t *handle) {
    if (!b || !handle) return set_error(FB_ERR_INVALID, "create_buffer: null argument");
    if (usage != FB_USAGE_WEIGHTS && usage != FB_USAGE_COMPUTE)
        return set_error(FB_ERR_INVALID, "create_buffer: bad usage %d", usage);
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    if (usage == FB_USAGE_COMPUTE) {
        // intermediates of any node whose activations live in this buffer fit
        // in its size plus a fixed margin (256-byte padding of each part)
        int rc = grow_scratch(b, size + (1u << 20));
        if (rc) return rc;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, size + kPad);
    b->device_allocs++;
    if (e != cudaSuccess) return cuda_fail(e, "create_buffer");
    e = cudaMemsetAsync(p, 0, size + kPad, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "create_buffer zero-fill");
    }
    const uint32_t h = b->next_handle++;
    b->buffers[h] = Buffer{static_cast<uint8_t *>(p), size, usage};
    *handle = h;
    return FB_OK;
}

int feml_b200_release_buffer(fb_backend *b, uint32_t handle) {
    if (!b) return set_error(FB_ERR_INVALID, "release_buffer: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    Buffer *buf;
    int rc = lookup(b, handle, "release_buffer", &buf);
    if (rc) return rc;
    DeviceGuard g(b->device);
    cudaStreamSynchronize(b->stream);  // queued work may still read it
    clear_plan_graphs(b);
    cudaFree(buf->ptr);
    b->buffers.erase(handle);
    return FB_OK;
}

int feml_b200_write(fb_backend *b, uint32_t h, uint64_t off, const void *src, uint64_t n) {
    if (!b || (!src && n)) return set_error(FB_ERR_INVALID, "write: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    Buffer *buf;
    int rc = lookup(b, h, "write", &buf);
    if (rc || (rc = check_range(*buf, h, off, n, "write"))) return rc;
    if (n == 0) return FB_OK;
    DeviceGuard g(b->device);
    cudaError_t e;
    if (n <= kStageBytes) {
        // the previous staged copy has left the staging area once this event is done
        e = cudaEventSynchronize(b->stage_free);
        if (e == cudaSuccess) {
            std::memcpy(b->stage, src, n);
            e = cudaMemcpyAsync(buf->ptr + off, b->stage, n, cudaMemcpyHostToDevice, b->stream);
        }
        if (e == cudaSuccess) e = cudaEventRecord(b->stage_free, b->stream);
        return e == cudaSuccess ? FB_OK : cuda_fail(e, "write");
    }
    e = cudaMemcpyAsync(buf->ptr + off, src, n, cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    return e == cudaSuccess ? FB_OK : cuda_fail(e, "write");
}

int feml_b200_buffer_from_host_ptr(fb_backend *b, const void *ptr, uint64_t size, uint64_t max_tensor_size,
                                   uint32_t *handle) {
    if (!b || !handle || (!ptr && size)) return set_error(FB_ERR_INVALID, "buffer_from_host_ptr: null argument");
    if (max_tensor_size > size)
        return set_error(FB_ERR_INVALID, "buffer_from_host_ptr: max_tensor_size %llu exceeds size %llu",
                         (unsigned long long)max_tensor_size, (unsigned long long)size);
    uint32_t h = 0;
    int rc = feml_b200_create_buffer(b, size, FB_USAGE_WEIGHTS, &h);
    if (rc) return rc;
    rc = feml_b200_write(b, h, 0, ptr, size);  // one DMA from the caller's pages
    if (rc) {
        const std::string msg = fb::last_error();
        feml_b200_release_buffer(b, h);
        return set_error(rc, "%s", msg.c_str());
    }
    *handle = h;
    return FB_OK;
}

int feml_b200_read(fb_backend *b, uint32_t h, uint64_t off, void *dst, uint64_t n) {
    if (!b || (!dst && n)) return set_error(FB_ERR_INVALID, "read: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    Buffer *buf;
    int rc = lookup(b, h, "read", &buf);
    if (rc || (rc = check_range(*buf, h, off, n, "read"))) return rc;
    if (n == 0) return FB_OK;
    DeviceGuard g(b->device);
    cudaError_t e = cudaMemcpyAsync(dst, buf->ptr + off, n, cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    return e == cudaSuccess ? FB_OK : cuda_fail(e, "read");
}

int feml_b200_fill(fb_backend *b, uint32_t h, uint64_t off, uint8_t value, uint64_t n) {
    if (!b) return set_error(FB_ERR_INVALID, "fill: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    Buffer *buf;
    int rc = lookup(b, h, "fill", &buf);
    if (rc || (rc = check_range(*buf, h, off, n, "fill"))) return rc;
    if (n == 0) return FB_OK;
    DeviceGuard g(b->device);
    cudaError_t e = cudaMemsetAsync(buf->ptr + off, value, n, b->stream);
    return e == cudaSuccess ? FB_OK : cuda_fail(e, "fill");
}

int feml_b200_synchronize(fb_backend *b) {
    if (!b) return set_error(FB_ERR_INVALID, "synchronize: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    cudaError_t e = cudaMemcpyAsync(b->status_host, b->status_dev, 4, cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return cuda_fail(e, "synchronize");
    const int32_t st = *b->status_host;
    if (st != 0) {
        cudaMemsetAsync(b->status_dev, 0, 4, b->stream);
        cudaStreamSynchronize(b->stream);
        if (st & fbk::STATUS_BAD_ID)
            return set_error(FB_ERR_DEVICE, "B200 backend error: mul_mat_id: expert id out of range (slots zeroed)");
        if (st & fbk::STATUS_TIMEOUT)
            return set_error(FB_ERR_DEVICE, "B200 backend error: a kernel wait timed out (results invalid)");
        return set_error(FB_ERR_DEVICE, "B200 backend error: kernel status 0x%x", (unsigned)st);
    }
    return FB_OK;
}

int feml_b200_supports_op(fb_backend *, int32_t op, const int32_t *dt, int32_t n) {
    switch (op) {
    case FB_OP_VIEW:
        return 1;  // zero-copy: nothing to execute
    case FB_OP_MUL_MAT:
        return n == 2 && dt && is_mul_mat_dtype(dt[0]) && dt[1] == FB_F32;
    case FB_OP_MUL_MAT_ID:
        return n == 3 && dt && is_weight_dtype(dt[0]) && dt[1] == FB_F32 && dt[2] == FB_I32;
    case FB_OP_RMS_NORM:
    case FB_OP_SILU:
        return n == 1 && dt && dt[0] == FB_F32;
    case FB_OP_ADD:
        return n == 2 && dt && dt[0] == FB_F32 && dt[1] == FB_F32;
    default:
        return 0;
    }
}

// Scratch bytes a node needs (0 for shapes the launch checks reject anyway).
uint64_t node_scratch(const fb_plan *plan, const fb_plan_tensor &node) {
    auto src = [&](int k) -> const fb_plan_tensor * {
        if (k >= node.n_srcs || node.srcs[k] < 0 || node.srcs[k] >= plan->n_tensors) return nullptr;
        return &plan->tensors[node.srcs[k]];
    };
    const fb_plan_tensor *w = src(0), *x = src(1);
    if (!w || !x || !is_mul_mat_dtype(w->dtype)) return 0;
    const int64_t K = w->ne[0], M = w->ne[1], N = x->ne[1];
    if (K <= 0 || M <= 0 || N <= 0 || K > (int64_t(1) << 31) || N > (int64_t(1) << 31)) return 0;
    if (node.op == FB_OP_MUL_MAT) return mul_mat_ws(w->dtype, K, M, N);
    const fb_plan_tensor *ids = src(2);
    if (node.op == FB_OP_MUL_MAT_ID && ids && ids->ne[0] > 0 && ids->ne[0] <= 1024 && w->ne[2] > 0)
        return id_ws_layout(nullptr, w->dtype, K, N, ids->ne[0], w->ne[2]).total;
    return 0;
}

}  // extern "C"

namespace {

// Every plan field the launches of graph_compute depend on, in a fixed order
// (buffers by handle: handles are never reused, and a buffer's address never
// changes while its handle lives).
template <typename F>
void visit_plan(const fb_plan *plan, F &&f) {
    f((uint64_t)plan->n_tensors);
    f((uint64_t)plan->n_nodes);
    f((uint64_t)plan->n_buffers);
    for (int64_t i = 0; i < plan->n_buffers; i++) {
        f((uint64_t)plan->buffers[i].handle);
        f(plan->buffers[i].size);
    }
    for (int64_t i = 0; i < plan->n_nodes; i++) f((uint64_t)plan->nodes[i]);
    for (int64_t i = 0; i < plan->n_tensors; i++) {
        const fb_plan_tensor &t = plan->tensors[i];
        f(((uint64_t)(uint32_t)t.op << 32) | (uint32_t)t.dtype);
        f(((uint64_t)t.op_params[0] << 32) | t.op_params[1]);
        f(((uint64_t)(uint32_t)t.n_srcs << 32) | t.flags);
        for (int k = 0; k < FB_MAX_SRC; k++) f((uint64_t)(int64_t)t.srcs[k]);
        f((uint64_t)(int64_t)t.buffer);
        f(t.offset);
        for (int d = 0; d < 4; d++) {
            f((uint64_t)t.ne[d]);
            f(t.nb[d]);
        }
    }
}

uint64_t plan_hash(const fb_plan *plan) {
    uint64_t h = 1469598103934665603ull;  // FNV-1a over the 64-bit fields
    visit_plan(plan, [&](uint64_t v) {
        h ^= v;
        h *= 1099511628211ull;
    });
    return h;
}

bool plan_matches(const std::vector<uint64_t> &key, const fb_plan *plan) {
    size_t i = 0;
    bool same = true;
    visit_plan(plan, [&](uint64_t v) {
        same = same && i < key.size() && key[i] == v;
        i++;
    });
    return same && i == key.size();
}

// Plans whose graphs are kept at once (a process that compiles many plans
// without releasing their buffers recaptures them after the cache is full).
constexpr size_t kMaxPlanGraphs = 256;

int run_nodes(fb_backend *b, const fb_plan *plan) {
    // add / silu nodes computed by the epilogue of the mul_mat before them
    std::vector<char> fused((size_t)plan->n_tensors, 0);
    std::vector<ActChain> chains((size_t)plan->n_nodes);
    for (int64_t i = 0; i < plan->n_nodes; i++) {
        const int64_t ti = plan->nodes[i];
        if (ti < 0 || ti >= plan->n_tensors) return set_error(FB_ERR_INVALID, "graph_compute: bad node index");
        if (plan->tensors[ti].op != FB_OP_MUL_MAT || fused[ti]) continue;
        chains[i] = act_chain(plan, i);
        if (chains[i].add >= 0) fused[chains[i].add] = 1;
        if (chains[i].silu >= 0) fused[chains[i].silu] = 1;
    }
    for (int64_t i = 0; i < plan->n_nodes; i++) {
        const int64_t ti = plan->nodes[i];
        const fb_plan_tensor &node = plan->tensors[ti];
        if (fused[ti]) continue;
        int rc;
        switch (node.op) {
        case FB_OP_VIEW:
            rc = FB_OK;
            break;
        case FB_OP_MUL_MAT:
            rc = compute_mul_mat(b, plan, node, chains[i].out >= 0 ? &chains[i] : nullptr);
            break;
        case FB_OP_ADD:
            rc = compute_add(b, plan, node);
            break;
        case FB_OP_SILU:
            rc = compute_silu(b, plan, node);
            break;
        case FB_OP_MUL_MAT_ID:
            rc = compute_mul_mat_id(b, plan, node);
            break;
        case FB_OP_RMS_NORM:
            rc = rms_fused(plan, ti) ? FB_OK : compute_rms_norm(b, plan, node);
            break;
        default:
            rc = set_error(FB_ERR_UNSUPPORTED, "B200: op %s not implemented", fb::op_name(node.op));
        }
        if (rc) return rc;
    }
    return FB_OK;
}

// Capture the launches of `plan` into a CUDA graph (without executing them)
// and cache it under `h`. Relaxed capture mode: the launchers may set kernel
// attributes or load modules on their first use. A capture that fails is
// cached as a node-by-node plan when `remember_failure`, else forgotten (the
// plan's first graph_compute then runs it node by node and captures again).
int capture_plan(fb_backend *b, const fb_plan *plan, uint64_t h, bool remember_failure) {
    if (b->graphs.size() >= kMaxPlanGraphs) {
        // bound the cache: wait for every launch of a cached graph, then drop them all
        const cudaError_t se = cudaStreamSynchronize(b->stream);
        if (se != cudaSuccess) return cuda_fail(se, "plan graph cache");
        clear_plan_graphs(b);
    }
    fb_backend::PlanGraph entry;
    visit_plan(plan, [&](uint64_t v) { entry.key.push_back(v); });
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeRelaxed);
    if (e == cudaSuccess) {
        const int crc = run_nodes(b, plan);
        e = cudaStreamEndCapture(b->stream, &graph);
        if (crc == FB_OK && e == cudaSuccess && graph) e = cudaGraphInstantiate(&entry.exec, graph, 0);
        else entry.exec = nullptr;
        if (e != cudaSuccess) entry.exec = nullptr;
    }
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();  // a failed capture is not an error of the caller: the plan runs node by node
    if (entry.exec || remember_failure) b->graphs.emplace(h, std::move(entry));
    return FB_OK;
}

// Scratch bytes of the plan's largest node.
int plan_scratch(const fb_plan *plan, uint64_t *need) {
    *need = 0;
    for (int64_t i = 0; i < plan->n_nodes; i++) {
        const int64_t ti = plan->nodes[i];
        if (ti < 0 || ti >= plan->n_tensors) return set_error(FB_ERR_INVALID, "graph_compute: bad node index");
        *need = std::max(*need, node_scratch(plan, plan->tensors[ti]));
    }
    return FB_OK;
}

}  // namespace

extern "C" {

// Compile-time preparation (fb_graph_compile calls it through the vtable
// once the plan's buffers exist; other callers call it after compile): the
// scratch arena grows to the plan's largest node and the plan's launches are
// captured into a CUDA graph, so the plan's first graph_compute already
// allocates nothing and launches one graph.
int feml_b200_prepare_plan(fb_backend *b, const fb_plan *plan) {
    if (!b || !plan) return set_error(FB_ERR_INVALID, "prepare_plan: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    uint64_t need = 0;
    int rc = plan_scratch(plan, &need);
    if (rc) return rc;
    if (need > b->scratch_bytes && (rc = grow_scratch(b, need))) return rc;
    if (!b->use_graphs) return FB_OK;
    const uint64_t h = plan_hash(plan);
    auto it = b->graphs.find(h);
    if (it != b->graphs.end()) return FB_OK;
    return capture_plan(b, plan, h, false);
}

// Repeated graph_compute of one plan replays a CUDA graph of its launches.
// A plan prepared at compile (feml_b200_prepare_plan) has its graph and its
// scratch already; otherwise the first call runs the nodes one by one
// (sizing the scratch, which may then grow once with a device synchronize)
// and captures the same launches into a graph (not executed). Later calls of
// a plan with identical fields launch that graph: one launch instead of one
// or more per node, and no allocation. Releasing a buffer, or growing the
// scratch, drops the cached graphs (they hold addresses). A capture that
// fails leaves the plan on the node-by-node path.
int feml_b200_graph_compute(fb_backend *b, const fb_plan *plan) {
    if (!b || !plan) return set_error(FB_ERR_INVALID, "graph_compute: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    uint64_t need = 0;
    int rc = plan_scratch(plan, &need);
    if (rc) return rc;
    if (need > b->scratch_bytes && (rc = grow_scratch(b, need))) return rc;
    uint64_t h = 0;
    if (b->use_graphs) {
        h = plan_hash(plan);
        auto it = b->graphs.find(h);
        if (it != b->graphs.end() && plan_matches(it->second.key, plan)) {
            if (!it->second.exec) return run_nodes(b, plan);
            const cudaError_t e = cudaGraphLaunch(it->second.exec, b->stream);
            return e == cudaSuccess ? FB_OK : cuda_fail(e, "graph_compute: graph launch");
        }
    }
    rc = run_nodes(b, plan);
    if (rc || !b->use_graphs || b->graphs.count(h)) return rc;  // (a hash collision keeps the first plan's graph)
    return capture_plan(b, plan, h, true);
}

int feml_b200_plan_fused_nodes(fb_backend *b, const fb_plan *plan, int64_t *count) {
    if (!b || !plan || !count) return set_error(FB_ERR_INVALID, "plan_fused_nodes: null argument");
    int64_t n = 0;
    std::vector<char> fused((size_t)plan->n_tensors, 0);
    for (int64_t i = 0; i < plan->n_nodes; i++) {
        const int64_t ti = plan->nodes[i];
        if (ti < 0 || ti >= plan->n_tensors) return set_error(FB_ERR_INVALID, "plan_fused_nodes: bad node index");
        const fb_plan_tensor &t = plan->tensors[ti];
        if (t.op == FB_OP_RMS_NORM && rms_fused(plan, ti)) n++;
        if (t.op != FB_OP_MUL_MAT || fused[ti]) continue;
        const ActChain c = act_chain(plan, i);
        for (int64_t f : {c.add, c.silu})
            if (f >= 0) {
                fused[f] = 1;
                n++;
            }
    }
    *count = n;
    return FB_OK;
}

int feml_b200_set_plan_graphs(fb_backend *b, int32_t enable) {
    if (!b) return set_error(FB_ERR_INVALID, "set_plan_graphs: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return cuda_fail(e, "set_plan_graphs");
    clear_plan_graphs(b);
    b->use_graphs = enable != 0;
    return FB_OK;
}

int feml_b200_plan_graphs(fb_backend *b, int64_t *cached, int64_t *replayable) {
    if (!b) return set_error(FB_ERR_INVALID, "plan_graphs: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    int64_t n = 0, r = 0;
    for (auto &kv : b->graphs) {
        n++;
        r += kv.second.exec != nullptr;
    }
    if (cached) *cached = n;
    if (replayable) *replayable = r;
    return FB_OK;
}

int feml_b200_backend_vtable(fb_backend *b, fb_backend_vtable *vt) {
    if (!b || !vt) return set_error(FB_ERR_INVALID, "backend_vtable: null argument");
    vt->ctx = b;
    vt->name = vt_name;
    vt->create_buffer = vt_create;
    vt->release_buffer = vt_release;
    vt->write = vt_write;
    vt->read = vt_read;
    vt->fill = vt_fill;
    vt->synchronize = vt_sync;
    vt->graph_compute = vt_compute;
    vt->supports_op = vt_supports;
    vt->prepare_plan = vt_prepare;
    return FB_OK;
}

int feml_b200_buffer_device_ptr(fb_backend *b, uint32_t h, void **ptr, uint64_t *size) {
    if (!b || !ptr) return set_error(FB_ERR_INVALID, "buffer_device_ptr: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    Buffer *buf;
    int rc = lookup(b, h, "buffer_device_ptr", &buf);
    if (rc) return rc;
    *ptr = buf->ptr;
    if (size) *size = buf->size;
    return FB_OK;
}

int feml_b200_stream(fb_backend *b, void **stream) {
    if (!b || !stream) return set_error(FB_ERR_INVALID, "stream: null argument");
    *stream = b->stream;
    return FB_OK;
}

int feml_b200_scratch_bytes(fb_backend *b, uint64_t *bytes) {
    if (!b || !bytes) return set_error(FB_ERR_INVALID, "scratch_bytes: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    *bytes = b->scratch_bytes;
    return FB_OK;
}

int feml_b200_device_allocations(fb_backend *b, uint64_t *count) {
    if (!b || !count) return set_error(FB_ERR_INVALID, "device_allocations: null argument");
    std::lock_guard<std::mutex> lk(b->mu);
    *count = b->device_allocs;
    return FB_OK;
}

int feml_b200_reserve_scratch(fb_backend *b, uint64_t bytes) {
    if (!b) return set_error(FB_ERR_INVALID, "reserve_scratch: null backend");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    return grow_scratch(b, bytes);
}

// ---- kernel-level entry points --------------------------------------------
int feml_b200_quantize(int32_t dtype, const void *x, uint64_t x_row_stride, void *y, int64_t rows, int64_t k,
                       void *stream) {
    return fbk::launch_quantize_rows(dtype, x, x_row_stride, y, rows, k, static_cast<cudaStream_t>(stream));
}

int feml_b200_mul_mat_launches(int32_t wtype, int64_t K, int64_t M, int64_t N, int32_t *count) {
    if (!count) return set_error(FB_ERR_INVALID, "mul_mat_launches: null out");
    *count = 0;
    if (K < 0 || M < 0 || N < 0) return set_error(FB_ERR_INVALID, "mul_mat_launches: negative dimension");
    if (!is_mul_mat_dtype(wtype)) return set_error(FB_ERR_UNSUPPORTED, "mul_mat_launches: dtype %d", wtype);
    *count = mul_mat_launches(wtype, K, M, N);
    return FB_OK;
}

int feml_b200_mul_mat_workspace(int32_t wtype, int64_t K, int64_t M, int64_t N, uint64_t *bytes) {
    if (!bytes) return set_error(FB_ERR_INVALID, "mul_mat_workspace: null out");
    *bytes = mul_mat_ws(wtype, K, M, N);
    return FB_OK;
}

int feml_b200_mul_mat(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *dst,
                      uint64_t dst_nb1, int64_t K, int64_t M, int64_t N, void *workspace, uint64_t workspace_bytes,
                      void *stream) {
    return do_mul_mat(wtype, w, w_nb1, x, x_nb1, dst, dst_nb1, K, M, N, workspace, workspace_bytes, nullptr,
                      static_cast<cudaStream_t>(stream));
}

int feml_b200_mul_mat_id_workspace(int32_t wtype, int64_t K, int64_t M, int64_t N, int64_t n_selected,
                                   int64_t n_experts, uint64_t *bytes) {
    (void)M;
    if (!bytes) return set_error(FB_ERR_INVALID, "mul_mat_id_workspace: null out");
    *bytes = id_ws_layout(nullptr, wtype, K, N, n_selected, n_experts).total;
    return FB_OK;
}

int feml_b200_mul_mat_id(int32_t wtype, const void *w, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                         const void *x, uint64_t x_nb1, const int32_t *ids, uint64_t ids_nb1, int64_t n_selected,
                         void *dst, uint64_t dst_nb1, uint64_t dst_nb2, int64_t K, int64_t M, int64_t N,
                         void *workspace, uint64_t workspace_bytes, int32_t *status, void *stream) {
    return do_mul_mat_id(wtype, w, w_nb1, w_nb2, n_experts, 0, 1, x, x_nb1, ids, ids_nb1, n_selected, dst, dst_nb1,
                         dst_nb2, K, M, N, workspace, workspace_bytes, status, static_cast<cudaStream_t>(stream));
}

int feml_b200_mul_mat_peer(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1,
                           void *const *peer_dst0, void *const *peer_dst1, uint32_t *const *peer_flags,
                           int32_t n_peers, uint64_t dst_nb1, uint32_t *counter, const uint32_t *epoch, int64_t K,
                           int64_t M, int64_t N, int32_t *status, void *stream) {
    if (!w || !x || !peer_dst0 || !peer_dst1 || !peer_flags || !counter || !epoch)
        return set_error(FB_ERR_INVALID, "mul_mat_peer: null argument");
    if (n_peers < 1 || n_peers > fbk::kMaxPeers)
        return set_error(FB_ERR_INVALID, "mul_mat_peer: %d peers (1..%d)", n_peers, fbk::kMaxPeers);
    if (K <= 0 || M <= 0 || N < 1)
        return set_error(FB_ERR_INVALID, "mul_mat_peer: bad dimensions (every rank needs rows, it signals the step)");
    if (!is_weight_dtype(wtype) || wtype == FB_F32)
        return set_error(FB_ERR_UNSUPPORTED, "mul_mat_peer: quantized weights only");
    if (K % fb::dtype_traits(wtype)->block_size) return set_error(FB_ERR_SHAPE, "mul_mat_peer: K not a block multiple");
    if (!fbk::gemv_supported(wtype, K, N) || !fbk::gemv_fused_ok(K, N))
        return set_error(FB_ERR_UNSUPPORTED, "mul_mat_peer: needs the fused decode GEMV (N <= 8, N*K <= 16384)");
    fbk::PeerOut po{};
    po.n = n_peers;
    po.count = counter;
    po.epoch = epoch;
    for (int r = 0; r < n_peers; r++) {
        po.y[0][r] = static_cast<uint8_t *>(peer_dst0[r]);
        po.y[1][r] = static_cast<uint8_t *>(peer_dst1[r]);
        po.flag[r] = peer_flags[r];
    }
    return fbk::launch_gemv(wtype, w, w_nb1, x, x_nb1, nullptr, dst_nb1, K, M, N, nullptr, status,
                            static_cast<cudaStream_t>(stream), true, &po);
}

int feml_b200_mul_mat_id_peer_owned(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2,
                                    int64_t n_experts, int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1,
                                    const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, void *const *peer_dst0,
                                    void *const *peer_dst1, uint32_t *const *peer_flags, int32_t n_peers,
                                    uint64_t dst_nb1, uint64_t dst_nb2, int64_t owner_tokens, uint32_t *counter,
                                    const uint32_t *epoch, int64_t K, int64_t M, int64_t N, void *workspace,
                                    uint64_t workspace_bytes, int32_t *status, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!w_local || !x || !ids || !peer_dst0 || !peer_dst1 || !peer_flags || !counter || !epoch)
        return set_error(FB_ERR_INVALID, "mul_mat_id_peer: null argument");
    if (n_peers < 1 || n_peers > fbk::kMaxPeers || n_peers != n_shards || shard < 0 || shard >= n_shards)
        return set_error(FB_ERR_INVALID, "mul_mat_id_peer: %d peers for shard %ld of %ld", n_peers, (long)shard,
                         (long)n_shards);
    if (K <= 0 || M <= 0 || N <= 0 || n_selected < 1 || n_experts < 1)
        return set_error(FB_ERR_INVALID, "mul_mat_id_peer: bad dimensions");
    if (owner_tokens < 0 || (owner_tokens > 0 && owner_tokens * n_shards < N))
        return set_error(FB_ERR_INVALID, "mul_mat_id_peer: %ld tokens per owner cannot hold %ld tokens on %ld ranks",
                         (long)owner_tokens, (long)N, (long)n_shards);
    const int64_t n_local = fbk::local_experts(n_experts, shard, n_shards);
    if (n_local < 1) return set_error(FB_ERR_INVALID, "mul_mat_id_peer: every shard needs an expert (it signals)");
    if (!fbk::gemm_tc_supported(wtype, K, M, N * n_selected, w_local, w_nb1) || (w_nb2 & 15) ||
        ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15))
        return set_error(FB_ERR_UNSUPPORTED,
                         "mul_mat_id_peer: needs the tcgen05 GEMM (quantized, K %% 256 == 0, 16-byte aligned)");
    const IdWorkspace need = id_ws_layout(nullptr, wtype, K, N, n_selected, n_local);
    if (need.total > workspace_bytes)
        return set_error(FB_ERR_INVALID, "mul_mat_id_peer: workspace of %lu bytes needed, %lu given",
                         (unsigned long)need.total, (unsigned long)workspace_bytes);
    const IdWorkspace L = id_ws_layout(workspace, wtype, K, N, n_selected, n_local);
    fbk::PeerOut po{};
    po.n = n_peers;
    po.count = counter;
    po.epoch = epoch;
    po.owner_tokens = (int)owner_tokens;
    for (int r = 0; r < n_peers; r++) {
        po.y[0][r] = static_cast<uint8_t *>(peer_dst0[r]);
        po.y[1][r] = static_cast<uint8_t *>(peer_dst1[r]);
        po.flag[r] = peer_flags[r];
    }
    // invalid ids: every rank zeroes the slot in its own buffer of this step
    int rc = fbk::launch_moe_route(ids, ids_nb1, n_selected, N, n_experts, shard, n_shards, L.counts, L.offsets,
                                   L.rows, L.tile_start, fbk::gemm_tc_block_n(wtype, K), status, po.y[0][shard], dst_nb1,
                                   dst_nb2, M, s, po.y[1][shard], epoch, owner_tokens);
    if (rc) return rc;
    fbk::GroupMap g{};
    g.counts = L.counts;
    g.offsets = L.offsets;
    g.rows = L.rows;
    g.tile_start = L.tile_start;
    g.n_groups = (int32_t)n_local;
    g.n_selected = (int32_t)n_selected;
    g.w_group_stride = w_nb2;
    g.dst_nb1 = dst_nb1;
    g.dst_nb2 = dst_nb2;
    g.max_tiles = (int32_t)((n_selected * N + fbk::gemm_tc_block_n(wtype, K) - 1) / fbk::gemm_tc_block_n(wtype, K) + n_local);
    const fbk::XQ16 xa = fbk::xq16_carve(wtype, L.xq, K, N * n_selected);
    rc = fbk::launch_quantize_q8_f16(x, x_nb1, K, N, xa, &g, s, wtype);
    if (rc) return rc;
    return fbk::launch_gemm_tc(wtype, w_local, w_nb1, xa, K, M, N, nullptr, 0, &g, status, s, &po);
}

int feml_b200_mul_mat_id_peer(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                              int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1, const int32_t *ids,
                              uint64_t ids_nb1, int64_t n_selected, void *const *peer_dst0, void *const *peer_dst1,
                              uint32_t *const *peer_flags, int32_t n_peers, uint64_t dst_nb1, uint64_t dst_nb2,
                              uint32_t *counter, const uint32_t *epoch, int64_t K, int64_t M, int64_t N,
                              void *workspace, uint64_t workspace_bytes, int32_t *status, void *stream) {
    return feml_b200_mul_mat_id_peer_owned(wtype, w_local, w_nb1, w_nb2, n_experts, shard, n_shards, x, x_nb1, ids,
                                           ids_nb1, n_selected, peer_dst0, peer_dst1, peer_flags, n_peers, dst_nb1,
                                           dst_nb2, 0, counter, epoch, K, M, N, workspace, workspace_bytes, status,
                                           stream);
}

int feml_b200_ipc_export(const void *ptr, void *handle, uint64_t handle_bytes, uint64_t *offset) {
    if (!ptr || !handle || !offset || handle_bytes != sizeof(cudaIpcMemHandle_t))
        return set_error(FB_ERR_INVALID, "ipc_export: need a pointer and a %zu-byte handle buffer",
                         sizeof(cudaIpcMemHandle_t));
    // the allocation that holds ptr (a caching allocator hands out pieces of
    // larger cudaMalloc blocks; IPC shares whole blocks)
    using GetRange = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
    static GetRange get_range = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_range = reinterpret_cast<GetRange>(f);
    });
    if (!get_range) return set_error(FB_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_error(FB_ERR_INVALID, "ipc_export: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return set_error(FB_ERR_CUDA, "ipc_export: %s", cudaGetErrorString(e));
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base;
    return FB_OK;
}

int feml_b200_ipc_open(const void *handle, uint64_t handle_bytes, void **base) {
    if (!handle || !base || handle_bytes != sizeof(cudaIpcMemHandle_t))
        return set_error(FB_ERR_INVALID, "ipc_open: need a %zu-byte handle", sizeof(cudaIpcMemHandle_t));
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(FB_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(e));
    return FB_OK;
}

int feml_b200_ipc_close(void *base) {
    if (!base) return set_error(FB_ERR_INVALID, "ipc_close: null");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return set_error(FB_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
    return FB_OK;
}

int feml_b200_peer_wait(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, int32_t *status, void *stream) {
    return fbk::launch_peer_wait(flag, epoch, n_ranks, status, static_cast<cudaStream_t>(stream));
}

int feml_b200_peer_wait_timeout(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, uint64_t timeout_us,
                                int32_t *status, void *stream) {
    return fbk::launch_peer_wait(flag, epoch, n_ranks, status, static_cast<cudaStream_t>(stream), timeout_us);
}

int feml_b200_mul_mat_id_shard(int32_t wtype, const void *w_local, uint64_t w_nb1, uint64_t w_nb2, int64_t n_experts,
                               int64_t shard, int64_t n_shards, const void *x, uint64_t x_nb1, const int32_t *ids,
                               uint64_t ids_nb1, int64_t n_selected, void *dst, uint64_t dst_nb1, uint64_t dst_nb2,
                               int64_t K, int64_t M, int64_t N, void *workspace, uint64_t workspace_bytes,
                               int32_t *status, void *stream) {
    return do_mul_mat_id(wtype, w_local, w_nb1, w_nb2, n_experts, shard, n_shards, x, x_nb1, ids, ids_nb1, n_selected,
                         dst, dst_nb1, dst_nb2, K, M, N, workspace, workspace_bytes, status,
                         static_cast<cudaStream_t>(stream));
}

int feml_b200_moe_route(const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, int64_t N, int64_t n_experts,
                        int32_t *counts, int32_t *offsets, int32_t *rows, int32_t *status, void *stream) {
    if (!ids || !counts || !offsets || !rows) return set_error(FB_ERR_INVALID, "moe_route: null argument");
    return fbk::launch_moe_route(ids, ids_nb1, n_selected, N, n_experts, 0, 1, counts, offsets, rows, nullptr, 64,
                                 status, nullptr, 0, 0, 0,
                                 static_cast<cudaStream_t>(stream));
}

int feml_b200_block_dots(int32_t wtype, const void *w, uint64_t w_nb1, const void *xq, int64_t K, int64_t M,
                         int64_t N, int32_t *out, void *stream) {
    if (!w || !xq || !out) return set_error(FB_ERR_INVALID, "block_dots: null argument");
    return fbk::launch_block_dots(wtype, w, w_nb1, xq, K, M, N, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
