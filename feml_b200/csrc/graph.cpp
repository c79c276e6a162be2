// C++ mirror of feml-core's build/compile flow for callers without a Rust
// toolchain: GraphBuilder (feml-core/src/graph.rs), the ggml-alloc style
// MemoryPlanner (feml-core/src/planner.rs), Layout (feml-core/src/layout.rs)
// and GraphPlan tensor IO (feml-core/src/plan.rs).
//
// The planner's offsets are part of the drop-in contract (a Rust GraphPlan and
// a plan built here must place every tensor at the same byte offset), so the
// allocation steps follow planner.rs step for step: 32-byte alignment,
// first-fit over an unsorted free list whose split remainders go to the end,
// sort + coalesce on free, inplace reuse of a sole parent, views sharing their
// source. Validation follows graph.rs, with the mul_mat / mul_mat_id dtype and
// ids-shape relaxations this backend needs (documented at each builder).
#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "host_common.h"

namespace fb {

constexpr int kMaxDims = 4;
constexpr uint64_t kPlannerAlignment = 32;   // planner.rs:53
constexpr uint64_t kElementAlignment = 4;    // graph.rs:19

static std::atomic<uint32_t> g_next_tensor_id{1};  // tensor.rs:18

struct Shape {
    int64_t dims[kMaxDims] = {1, 1, 1, 1};
    int rank = 1;
};

struct Layout {
    Shape shape;
    uint64_t stride[kMaxDims] = {0, 0, 0, 0};
    uint64_t offset = 0;
};

struct TensorMeta {
    uint32_t id = 0;
    std::string name;
    int32_t dtype = FB_F32;
    Layout layout;
    int32_t op = FB_OP_NONE;
    uint32_t op_params[2] = {0, 0};
    std::vector<uint32_t> srcs;
    uint32_t view_src = 0;  // 0 = none
    uint32_t flags = 0;
};

static int make_shape(const int64_t *dims, int32_t rank, Shape *out) {
    if (rank < 1 && rank != 0) return set_error(FB_ERR_SHAPE, "shape error: negative rank");
    if (rank > kMaxDims)
        return set_error(FB_ERR_SHAPE, "shape error: rank %d exceeds MAX_DIMS = %d", rank, kMaxDims);
    Shape s;
    for (int i = 0; i < rank; i++) {
        if (dims[i] <= 0) return set_error(FB_ERR_SHAPE, "shape error: dimensions must be non-zero");
        s.dims[i] = dims[i];
    }
    s.rank = rank;
    *out = s;
    return FB_OK;
}

// Layout::new (layout.rs:32-48).
static int make_layout(int32_t dtype, const Shape &shape, Layout *out) {
    const DTypeTraits *t = dtype_traits(dtype);
    if (!t) return set_error(FB_ERR_INVALID, "unknown dtype %d", dtype);
    Layout l;
    l.shape = shape;
    l.stride[0] = (uint64_t)t->type_size;
    l.stride[1] = l.stride[0] * (uint64_t)(shape.dims[0] / t->block_size);
    for (int i = 2; i < kMaxDims; i++) l.stride[i] = l.stride[i - 1] * (uint64_t)shape.dims[i - 1];
    *out = l;
    return FB_OK;
}

// Layout::nbytes (layout.rs:51-60).
static uint64_t layout_nbytes(const Layout &l, int32_t dtype) {
    const DTypeTraits *t = dtype_traits(dtype);
    uint64_t bytes = (uint64_t)(l.shape.dims[0] * t->type_size / t->block_size);
    for (int i = 1; i < kMaxDims; i++) bytes += (uint64_t)(l.shape.dims[i] - 1) * l.stride[i];
    return bytes;
}

static bool can_inplace(int32_t op) {  // op.rs:98-110
    switch (op) {
    case FB_OP_MUL: case FB_OP_ADD: case FB_OP_RMS_NORM: case FB_OP_SILU: case FB_OP_SOFTMAX:
    case FB_OP_ROPE: case FB_OP_DIAG_MASK_INF: case FB_OP_SCALE:
        return true;
    default:
        return false;
    }
}

static bool is_matmul_id_weight_dtype(int32_t d) {
    return d == FB_F32 || d == FB_Q8_0 || d == FB_Q4_0 || d == FB_Q4_K;
}

static bool is_matmul_weight_dtype(int32_t d) {
    return is_matmul_id_weight_dtype(d) || d == FB_Q5_K || d == FB_Q6_K;
}

// ---------------------------------------------------------------------------
// Planner (planner.rs)
// ---------------------------------------------------------------------------
enum Kind { kWeights = 0, kCompute = 1 };

struct Assignment {
    int kind;
    uint64_t offset;
};

static uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct Talloc {  // planner.rs:55-101
    uint64_t used = 0;
    std::vector<std::pair<uint64_t, uint64_t>> free_list;  // (offset, size)

    uint64_t alloc(uint64_t size) {
        size = align_up(size, kPlannerAlignment);
        for (size_t i = 0; i < free_list.size(); i++) {
            if (free_list[i].second >= size) {
                const uint64_t offset = free_list[i].first, free_size = free_list[i].second;
                free_list.erase(free_list.begin() + (long)i);
                if (free_size > size) free_list.push_back({offset + size, free_size - size});
                return offset;
            }
        }
        const uint64_t offset = align_up(used, kPlannerAlignment);
        used = offset + size;
        return offset;
    }

    void release(uint64_t offset, uint64_t size) {
        free_list.push_back({offset, align_up(size, kPlannerAlignment)});
        std::sort(free_list.begin(), free_list.end());
        std::vector<std::pair<uint64_t, uint64_t>> merged;
        for (auto &fr : free_list) {
            if (!merged.empty() && merged.back().first + merged.back().second == fr.first) {
                merged.back().second += fr.second;
                continue;
            }
            merged.push_back(fr);
        }
        free_list.swap(merged);
    }
};

struct PlannerOutput {
    std::map<uint32_t, Assignment> assignments;
    uint64_t weights_size = 0, compute_size = 0;
};

static int kind_of(const TensorMeta &t) { return (t.flags & FB_FLAG_WEIGHT) ? kWeights : kCompute; }

struct Planner {
    const std::vector<TensorMeta> &tensors;
    std::map<uint32_t, size_t> by_id;
    Talloc tallocs[2];
    std::map<uint32_t, Assignment> assigned;
    std::map<uint32_t, bool> allocated;

    explicit Planner(const std::vector<TensorMeta> &t) : tensors(t) {
        for (size_t i = 0; i < t.size(); i++) by_id[t[i].id] = i;
    }

    const TensorMeta *at(uint32_t id) const {
        auto it = by_id.find(id);
        return it == by_id.end() ? nullptr : &tensors[it->second];
    }

    uint64_t nbytes(const TensorMeta &t) const { return layout_nbytes(t.layout, t.dtype); }

    // planner.rs:118-143
    int allocate(uint32_t id) {
        const TensorMeta *t = at(id);
        if (!t) return set_error(FB_ERR_INVALID, "planner: tensor %u is not reachable", id);
        if (allocated[id]) return FB_OK;
        if (t->view_src) {
            int rc = allocate(t->view_src);
            if (rc) return rc;
            const Assignment a = assigned.at(t->view_src);
            assigned[id] = {a.kind, a.offset + t->layout.offset};
            allocated[id] = true;
            return FB_OK;
        }
        const int kind = kind_of(*t);
        assigned[id] = {kind, tallocs[kind].alloc(nbytes(*t))};
        allocated[id] = true;
        return FB_OK;
    }

    // planner.rs:156-261
    int run(const std::vector<size_t> &order, PlannerOutput *out) {
        std::map<uint32_t, int64_t> children, views;
        for (auto &t : tensors) { children[t.id] = 0; views[t.id] = 0; allocated[t.id] = false; }
        for (auto &t : tensors) {
            if (t.view_src) {
                if (!views.count(t.view_src))
                    return set_error(FB_ERR_INVALID, "planner: view source %u is not reachable", t.view_src);
                views[t.view_src] += 1;
            }
            for (uint32_t s : t.srcs) {
                if (!children.count(s)) return set_error(FB_ERR_INVALID, "planner: source %u is not reachable", s);
                children[s] += 1;
            }
        }
        std::map<uint32_t, int64_t> live_children = children, live_views = views;
        for (auto &t : tensors) {
            if (t.flags & (FB_FLAG_INPUT | FB_FLAG_WEIGHT)) {
                int rc = allocate(t.id);
                if (rc) return rc;
            }
        }
        for (size_t idx : order) {
            const TensorMeta &node = tensors[idx];
            if (node.view_src) {
                int rc = allocate(node.view_src);
                if (rc) return rc;
                const Assignment a = assigned.at(node.view_src);
                assigned[node.id] = {a.kind, a.offset + node.layout.offset};
                allocated[node.id] = true;
            } else {
                for (uint32_t s : node.srcs) {
                    if (!allocated[s]) {
                        int rc = allocate(s);
                        if (rc) return rc;
                    }
                }
                bool reused = false;
                if (can_inplace(node.op)) {
                    for (uint32_t s : node.srcs) {
                        const TensorMeta &parent = *at(s);
                        const bool ok = allocated[s] && live_children[s] == 1 && live_views[s] == 0 &&
                                        !(parent.flags & FB_FLAG_OUTPUT) && !(parent.flags & FB_FLAG_WEIGHT) &&
                                        node.dtype == parent.dtype &&
                                        std::equal(node.layout.shape.dims, node.layout.shape.dims + kMaxDims,
                                                   parent.layout.shape.dims) &&
                                        node.layout.shape.rank == parent.layout.shape.rank &&
                                        std::equal(node.layout.stride, node.layout.stride + kMaxDims,
                                                   parent.layout.stride);
                        if (ok) {
                            assigned[node.id] = assigned.at(s);
                            allocated[node.id] = true;
                            allocated[s] = false;
                            reused = true;
                            break;
                        }
                    }
                }
                if (!reused) {
                    const int kind = kind_of(node);
                    assigned[node.id] = {kind, tallocs[kind].alloc(nbytes(node))};
                    allocated[node.id] = true;
                }
            }
            for (uint32_t s : node.srcs) {
                live_children[s] -= 1;
                const TensorMeta &parent = *at(s);
                const bool never_freed = parent.flags & (FB_FLAG_INPUT | FB_FLAG_WEIGHT | FB_FLAG_OUTPUT);
                if (live_children[s] == 0 && live_views[s] == 0 && !never_freed) {
                    if (allocated[s]) {
                        const Assignment a = assigned.at(s);
                        tallocs[a.kind].release(a.offset, nbytes(parent));
                        allocated[s] = false;
                    } else if (parent.view_src) {
                        const uint32_t vs = parent.view_src;
                        live_views[vs] -= 1;
                        const TensorMeta &vt = *at(vs);
                        if (live_views[vs] == 0 && live_children[vs] == 0 && !(vt.flags & FB_FLAG_OUTPUT) &&
                            allocated[vs]) {
                            const Assignment a = assigned.at(vs);
                            tallocs[a.kind].release(a.offset, nbytes(vt));
                            allocated[vs] = false;
                        }
                    }
                }
            }
        }
        out->assignments = assigned;
        out->weights_size = tallocs[kWeights].used;
        out->compute_size = tallocs[kCompute].used;
        return FB_OK;
    }
};

// ---------------------------------------------------------------------------
// GraphBuilder (graph.rs)
// ---------------------------------------------------------------------------
struct Graph {
    std::vector<TensorMeta> tensors;
    std::map<uint32_t, size_t> by_id;
    std::vector<uint32_t> outputs;

    TensorMeta *get(uint32_t id) {
        auto it = by_id.find(id);
        return it == by_id.end() ? nullptr : &tensors[it->second];
    }

    uint32_t push(TensorMeta m) {
        const uint32_t id = m.id;
        by_id[id] = tensors.size();
        tensors.push_back(std::move(m));
        return id;
    }

    int new_meta(const char *name, int32_t dtype, const Shape &shape, TensorMeta *m) {
        TensorMeta t;
        int rc = make_layout(dtype, shape, &t.layout);
        if (rc) return rc;
        t.id = g_next_tensor_id.fetch_add(1);
        t.name = name ? name : "";
        t.dtype = dtype;
        *m = std::move(t);
        return FB_OK;
    }

    int leaf(const char *name, int32_t dtype, const int64_t *dims, int32_t rank, uint32_t flag, uint32_t *id) {
        Shape s;
        int rc = make_shape(dims, rank, &s);
        if (rc) return rc;
        TensorMeta m;
        rc = new_meta(name, dtype, s, &m);
        if (rc) return rc;
        m.flags |= flag;
        *id = push(std::move(m));
        return FB_OK;
    }

    // graph.rs:262-273
    int pair(uint32_t a, uint32_t b, const char *op, TensorMeta **ma, TensorMeta **mb) {
        *ma = get(a);
        if (!*ma) return set_error(FB_ERR_INVALID, "%s: unknown tensor %u", op, a);
        *mb = get(b);
        if (!*mb) return set_error(FB_ERR_INVALID, "%s: unknown tensor %u", op, b);
        if ((*ma)->dtype != (*mb)->dtype)
            return set_error(FB_ERR_SHAPE, "shape error: %s: dtype mismatch: %s vs %s", op,
                             dtype_traits((*ma)->dtype)->name, dtype_traits((*mb)->dtype)->name);
        return FB_OK;
    }

    int node(int32_t op, const char *name, int32_t dtype, const Shape &shape, std::vector<uint32_t> srcs,
             uint32_t *id) {
        TensorMeta m;
        int rc = new_meta(name, dtype, shape, &m);
        if (rc) return rc;
        m.op = op;
        m.srcs = std::move(srcs);
        *id = push(std::move(m));
        return FB_OK;
    }

    // op.rs:118-143 (trailing dims align)
    static int broadcast(const Shape &a, const Shape &b, Shape *out) {
        const int rank = std::max(a.rank, b.rank);
        int64_t dims[kMaxDims] = {1, 1, 1, 1};
        for (int back = 0; back < rank; back++) {
            const int64_t da = back < a.rank ? a.dims[a.rank - 1 - back] : 1;
            const int64_t db = back < b.rank ? b.dims[b.rank - 1 - back] : 1;
            int64_t d;
            if (da == db) d = da;
            else if (da == 1) d = db;
            else if (db == 1) d = da;
            else return set_error(FB_ERR_SHAPE, "shape error: cannot broadcast dim %d: %ld vs %ld", rank - 1 - back,
                                  (long)da, (long)db);
            dims[rank - 1 - back] = d;
        }
        return make_shape(dims, rank, out);
    }

    int elementwise(int32_t op, const char *name, uint32_t a, uint32_t b, uint32_t *id) {
        TensorMeta *ma, *mb;
        int rc = pair(a, b, name, &ma, &mb);
        if (rc) return rc;
        Shape s;
        rc = broadcast(ma->layout.shape, mb->layout.shape, &s);
        if (rc) return rc;
        return node(op, name, ma->dtype, s, {a, b}, id);
    }

    int unary(int32_t op, const char *name, uint32_t x, uint32_t *id) {
        TensorMeta *mx = get(x);
        if (!mx) return set_error(FB_ERR_INVALID, "%s: unknown tensor %u", name, x);
        return node(op, name, mx->dtype, mx->layout.shape, {x}, id);
    }

    // graph.rs:140-142 (unary; Op::RmsNorm { eps }, op.rs:26): eps travels in
    // op_params[0] as f32 bits.
    int rms_norm(uint32_t x, float eps, uint32_t *id) {
        int rc = unary(FB_OP_RMS_NORM, "rms_norm", x, id);
        if (rc) return rc;
        uint32_t bits;
        std::memcpy(&bits, &eps, 4);
        get(*id)->op_params[0] = bits;
        return FB_OK;
    }

    // graph.rs:89-108
    int view(uint32_t src, uint64_t offset, const int64_t *dims, int32_t rank, uint32_t *id) {
        TensorMeta *ms = get(src);
        if (!ms) return set_error(FB_ERR_INVALID, "view: unknown source");
        const uint64_t src_bytes = layout_nbytes(ms->layout, ms->dtype);
        const int32_t dtype = ms->dtype;
        Shape s;
        int rc = make_shape(dims, rank, &s);
        if (rc) return rc;
        TensorMeta m;
        rc = new_meta("view", dtype, s, &m);
        if (rc) return rc;
        if (offset % kElementAlignment != 0)
            return set_error(FB_ERR_SHAPE, "shape error: view: offset %lu is not %lu-byte aligned",
                             (unsigned long)offset, (unsigned long)kElementAlignment);
        const uint64_t vb = layout_nbytes(m.layout, dtype);
        if (offset + vb > src_bytes)
            return set_error(FB_ERR_SHAPE, "shape error: view: offset %lu + %lu > source bytes %lu",
                             (unsigned long)offset, (unsigned long)vb, (unsigned long)src_bytes);
        m.op = FB_OP_VIEW;
        m.view_src = src;
        m.layout.offset = offset;
        *id = push(std::move(m));
        return FB_OK;
    }

    // graph.rs:122-138, relaxed for quantized weights: src0 in {F32, Q8_0,
    // Q4_0, Q4_K, Q5_K, Q6_K} with src1 F32 (the dtype-equality rule of pair() does not
    // apply), output F32 instead of src0's dtype, ne0 % block_size(src0) == 0.
    int mul_mat(uint32_t a, uint32_t b, uint32_t *id) {
        TensorMeta *ma = get(a);
        if (!ma) return set_error(FB_ERR_INVALID, "mul_mat: unknown tensor %u", a);
        TensorMeta *mb = get(b);
        if (!mb) return set_error(FB_ERR_INVALID, "mul_mat: unknown tensor %u", b);
        if (!is_matmul_weight_dtype(ma->dtype))
            return set_error(FB_ERR_UNSUPPORTED, "dtype %s not supported for op mul_mat", dtype_traits(ma->dtype)->name);
        if (mb->dtype != FB_F32)
            return set_error(FB_ERR_UNSUPPORTED, "dtype %s not supported for op mul_mat", dtype_traits(mb->dtype)->name);
        if (ma->layout.shape.dims[0] != mb->layout.shape.dims[0])
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat: inner dim mismatch: %ld vs %ld",
                             (long)ma->layout.shape.dims[0], (long)mb->layout.shape.dims[0]);
        if (ma->layout.shape.rank > 2 || mb->layout.shape.rank > 2)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat: rank > 2 not supported yet");
        const int64_t blk = dtype_traits(ma->dtype)->block_size;
        if (ma->layout.shape.dims[0] % blk != 0)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat: inner dim %ld is not a multiple of the %s block size %ld",
                             (long)ma->layout.shape.dims[0], dtype_traits(ma->dtype)->name, (long)blk);
        const int64_t dims[2] = {ma->layout.shape.dims[1], mb->layout.shape.dims[1]};
        Shape s;
        int rc = make_shape(dims, 2, &s);
        if (rc) return rc;
        return node(FB_OP_MUL_MAT, "mul_mat", FB_F32, s, {a, b}, id);
    }

    // graph.rs:215-250 with ggml semantics: ids I32 [n_selected, N] (the
    // reference declares [n_experts, N]), output [M, n_selected, N] F32.
    int mul_mat_id(uint32_t w, uint32_t x, uint32_t ids, uint32_t n_selected, uint32_t *id) {
        TensorMeta *mw = get(w);
        if (!mw) return set_error(FB_ERR_INVALID, "mul_mat_id: unknown weights");
        TensorMeta *mx = get(x);
        if (!mx) return set_error(FB_ERR_INVALID, "mul_mat_id: unknown x");
        TensorMeta *mi = get(ids);
        if (!mi) return set_error(FB_ERR_INVALID, "mul_mat_id: unknown ids");
        if (!is_matmul_id_weight_dtype(mw->dtype))
            return set_error(FB_ERR_UNSUPPORTED, "dtype %s not supported for op mul_mat_id", dtype_traits(mw->dtype)->name);
        if (mx->dtype != FB_F32)
            return set_error(FB_ERR_UNSUPPORTED, "dtype %s not supported for op mul_mat_id", dtype_traits(mx->dtype)->name);
        if (mi->dtype != FB_I32) return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: ids must be i32");
        if (mw->layout.shape.dims[0] != mx->layout.shape.dims[0])
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: inner dim mismatch");
        if (mw->layout.shape.rank > 3 || mx->layout.shape.rank > 2 || mi->layout.shape.rank > 2)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: rank not supported");
        const int64_t blk = dtype_traits(mw->dtype)->block_size;
        if (mw->layout.shape.dims[0] % blk != 0)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: inner dim is not a multiple of the block size");
        const int64_t n_experts = mw->layout.shape.dims[2];
        if (n_selected == 0 || (int64_t)n_selected > n_experts)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: n_selected %u not in [1, %ld]", n_selected,
                             (long)n_experts);
        if (mi->layout.shape.dims[0] != (int64_t)n_selected)
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: ids rows %ld != n_selected %u",
                             (long)mi->layout.shape.dims[0], n_selected);
        if (mi->layout.shape.dims[1] != mx->layout.shape.dims[1])
            return set_error(FB_ERR_SHAPE, "shape error: mul_mat_id: ids cols != x cols");
        const int64_t dims[3] = {mw->layout.shape.dims[1], (int64_t)n_selected, mx->layout.shape.dims[1]};
        Shape s;
        int rc = make_shape(dims, 3, &s);
        if (rc) return rc;
        rc = node(FB_OP_MUL_MAT_ID, "mul_mat_id", FB_F32, s, {w, x, ids}, id);
        if (rc) return rc;
        TensorMeta *out = get(*id);
        out->op_params[0] = (uint32_t)n_experts;
        out->op_params[1] = n_selected;
        return FB_OK;
    }

    int mark_output(uint32_t id) {  // graph.rs:57-65
        TensorMeta *t = get(id);
        if (!t) return set_error(FB_ERR_INVALID, "mark_output: unknown tensor");
        t->flags |= FB_FLAG_OUTPUT;
        outputs.push_back(id);
        return FB_OK;
    }

    // graph.rs:302-333: iterative DFS post-order from the outputs.
    int topo_order(std::vector<size_t> *order, std::set<uint32_t> *reachable) {
        std::vector<std::pair<size_t, bool>> stack;
        for (uint32_t out : outputs) {
            auto it = by_id.find(out);
            if (it == by_id.end()) return set_error(FB_ERR_INVALID, "output tensor %u not in graph", out);
            stack.push_back({it->second, false});
        }
        while (!stack.empty()) {
            auto [idx, expanded] = stack.back();
            stack.pop_back();
            const TensorMeta &t = tensors[idx];
            if (expanded) {
                if (t.op != FB_OP_NONE) order->push_back(idx);
                continue;
            }
            if (reachable->count(t.id)) continue;
            reachable->insert(t.id);
            stack.push_back({idx, true});
            for (uint32_t s : t.srcs) {
                auto it = by_id.find(s);
                if (it != by_id.end()) stack.push_back({it->second, false});
            }
        }
        return FB_OK;
    }

    uint64_t uid(const std::vector<size_t> &order) const {  // graph.rs:335-347 (FNV-1a 64)
        uint64_t h = 1469598103934665603ull;
        for (size_t i : order) {
            const TensorMeta &t = tensors[i];
            h ^= (uint64_t)t.id;
            h *= 1099511628211ull;
            for (uint32_t s : t.srcs) {
                h ^= (uint64_t)s;
                h *= 1099511628211ull;
            }
        }
        return h;
    }
};

}  // namespace fb

// ---------------------------------------------------------------------------
// Compiled plan
// ---------------------------------------------------------------------------
struct fb_graph {
    fb::Graph g;
};

struct fb_compiled_plan {
    std::vector<fb_plan_tensor> tensors;
    std::vector<int64_t> nodes;
    std::vector<fb_plan_buffer> buffers;
    fb_plan view;
    bool released = false;
};

using namespace fb;

static int vt_error(const fb_backend_vtable *vt, int rc, const char *what) {
    (void)vt;
    (void)what;
    return rc;  // the backend already recorded its message
}

extern "C" {

int fb_graph_new(fb_graph **out) {
    if (!out) return set_error(FB_ERR_INVALID, "fb_graph_new: null out");
    try {
        *out = new fb_graph();
    } catch (...) {
        return set_error(FB_ERR_INVALID, "fb_graph_new: out of host memory");
    }
    return FB_OK;
}

void fb_graph_free(fb_graph *g) { delete g; }

#define GRAPH_GUARD(g)                                                          \
    if (!(g)) return set_error(FB_ERR_INVALID, "null graph");                   \
    try {
#define GRAPH_END                                                               \
    }                                                                           \
    catch (const std::exception &e) {                                           \
        return set_error(FB_ERR_INVALID, "host exception: %s", e.what());       \
    }

int fb_graph_input(fb_graph *g, const char *name, int32_t dtype, const int64_t *dims, int32_t rank, uint32_t *id) {
    GRAPH_GUARD(g)
    if (!id) return set_error(FB_ERR_INVALID, "null id");
    return g->g.leaf(name, dtype, dims, rank, FB_FLAG_INPUT, id);
    GRAPH_END
}

int fb_graph_weight(fb_graph *g, const char *name, int32_t dtype, const int64_t *dims, int32_t rank, uint32_t *id) {
    GRAPH_GUARD(g)
    if (!id) return set_error(FB_ERR_INVALID, "null id");
    return g->g.leaf(name, dtype, dims, rank, FB_FLAG_WEIGHT, id);
    GRAPH_END
}

int fb_graph_view(fb_graph *g, uint32_t src, uint64_t offset, const int64_t *dims, int32_t rank, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.view(src, offset, dims, rank, id);
    GRAPH_END
}

int fb_graph_mul(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.elementwise(FB_OP_MUL, "mul", a, b, id);
    GRAPH_END
}

int fb_graph_add(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.elementwise(FB_OP_ADD, "add", a, b, id);
    GRAPH_END
}

int fb_graph_silu(fb_graph *g, uint32_t x, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.unary(FB_OP_SILU, "silu", x, id);
    GRAPH_END
}

int fb_graph_rms_norm(fb_graph *g, uint32_t x, float eps, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.rms_norm(x, eps, id);
    GRAPH_END
}

int fb_graph_copy(fb_graph *g, uint32_t x, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.unary(FB_OP_COPY, "copy", x, id);
    GRAPH_END
}

int fb_graph_mul_mat(fb_graph *g, uint32_t a, uint32_t b, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.mul_mat(a, b, id);
    GRAPH_END
}

int fb_graph_mul_mat_id(fb_graph *g, uint32_t w, uint32_t x, uint32_t ids, uint32_t n_selected, uint32_t *id) {
    GRAPH_GUARD(g)
    return g->g.mul_mat_id(w, x, ids, n_selected, id);
    GRAPH_END
}

int fb_graph_mark_output(fb_graph *g, uint32_t id) {
    GRAPH_GUARD(g)
    return g->g.mark_output(id);
    GRAPH_END
}

int fb_graph_tensor_info(fb_graph *g, uint32_t id, int32_t *dtype, int64_t *ne, uint64_t *nb, uint32_t *flags,
                         int32_t *op) {
    GRAPH_GUARD(g)
    TensorMeta *t = g->g.get(id);
    if (!t) return set_error(FB_ERR_INVALID, "unknown tensor %u", id);
    if (dtype) *dtype = t->dtype;
    for (int i = 0; i < 4; i++) {
        if (ne) ne[i] = t->layout.shape.dims[i];
        if (nb) nb[i] = t->layout.stride[i];
    }
    if (flags) *flags = t->flags;
    if (op) *op = t->op;
    return FB_OK;
    GRAPH_END
}

// graph.rs:349-442
int fb_graph_compile(fb_graph *gh, const fb_backend_vtable *be, fb_compiled_plan **out) {
    GRAPH_GUARD(gh)
    if (!be || !out) return set_error(FB_ERR_INVALID, "compile: null backend or out");
    Graph &g = gh->g;
    if (g.outputs.empty()) return set_error(FB_ERR_INVALID, "compile: no outputs marked");
    std::vector<size_t> order;
    std::set<uint32_t> reachable;
    int rc = g.topo_order(&order, &reachable);
    if (rc) return rc;
    const uint64_t uid = g.uid(order);

    // Fail fast: reject unsupported ops before allocating any buffer.
    for (size_t i : order) {
        const TensorMeta &n = g.tensors[i];
        std::vector<int32_t> dts;
        for (uint32_t s : n.srcs) dts.push_back(g.tensors[g.by_id.at(s)].dtype);
        if (!be->supports_op(be->ctx, n.op, dts.data(), (int32_t)dts.size()))
            return set_error(FB_ERR_UNSUPPORTED, "compile: backend '%s' does not support op %s", be->name(be->ctx),
                             op_name(n.op));
    }

    std::vector<TensorMeta> reach;
    for (auto &t : g.tensors)
        if (reachable.count(t.id)) reach.push_back(t);
    std::vector<size_t> order_rel;
    for (size_t i : order) {
        const uint32_t id = g.tensors[i].id;
        for (size_t j = 0; j < reach.size(); j++)
            if (reach[j].id == id) { order_rel.push_back(j); break; }
    }
    Planner planner(reach);
    PlannerOutput po;
    rc = planner.run(order_rel, &po);
    if (rc) return rc;

    std::unique_ptr<fb_compiled_plan> plan(new fb_compiled_plan());
    int buffer_idx[2] = {-1, -1};
    const uint64_t sizes[2] = {po.weights_size, po.compute_size};
    for (int kind = 0; kind < 2; kind++) {  // BUFFER_KINDS order: Weights, Compute
        if (sizes[kind] == 0) continue;
        uint32_t h = 0;
        rc = be->create_buffer(be->ctx, sizes[kind], kind == kWeights ? FB_USAGE_WEIGHTS : FB_USAGE_COMPUTE, &h);
        if (rc) {
            for (auto &b : plan->buffers) be->release_buffer(be->ctx, b.handle);
            return vt_error(be, rc, "create_buffer");
        }
        buffer_idx[kind] = (int)plan->buffers.size();
        plan->buffers.push_back({h, sizes[kind], kind == kWeights ? FB_USAGE_WEIGHTS : FB_USAGE_COMPUTE});
    }
    if (plan->buffers.empty()) return set_error(FB_ERR_INVALID, "compile: graph has no memory requirements");

    // Leafs first (weights before other leafs, stable), then nodes in builder order.
    std::vector<const TensorMeta *> seq;
    for (auto &t : reach)
        if (t.op == FB_OP_NONE && (t.flags & FB_FLAG_WEIGHT)) seq.push_back(&t);
    for (auto &t : reach)
        if (t.op == FB_OP_NONE && !(t.flags & FB_FLAG_WEIGHT)) seq.push_back(&t);
    for (auto &t : reach)
        if (t.op != FB_OP_NONE) seq.push_back(&t);
    std::map<uint32_t, int64_t> tidx;
    for (const TensorMeta *t : seq) {
        fb_plan_tensor pt;
        memset(&pt, 0, sizeof(pt));
        pt.id = t->id;
        pt.op = t->op;
        pt.op_params[0] = t->op_params[0];
        pt.op_params[1] = t->op_params[1];
        int ns = 0;
        for (uint32_t s : t->srcs) {
            auto it = tidx.find(s);
            if (it != tidx.end() && ns < FB_MAX_SRC) pt.srcs[ns++] = (int32_t)it->second;
        }
        pt.n_srcs = ns;
        auto a = po.assignments.find(t->id);
        if (a == po.assignments.end()) {
            for (auto &b : plan->buffers) be->release_buffer(be->ctx, b.handle);
            return set_error(FB_ERR_INVALID, "compile: tensor %u has no allocation", t->id);
        }
        pt.buffer = buffer_idx[a->second.kind];
        pt.offset = a->second.offset;
        pt.dtype = t->dtype;
        pt.flags = t->flags;
        for (int i = 0; i < 4; i++) {
            pt.ne[i] = t->layout.shape.dims[i];
            pt.nb[i] = t->layout.stride[i];
        }
        tidx[t->id] = (int64_t)plan->tensors.size();
        plan->tensors.push_back(pt);
    }
    for (size_t i : order) plan->nodes.push_back(tidx.at(g.tensors[i].id));
    plan->view.uid = uid;
    plan->view.tensors = plan->tensors.data();
    plan->view.n_tensors = (int64_t)plan->tensors.size();
    plan->view.nodes = plan->nodes.data();
    plan->view.n_nodes = (int64_t)plan->nodes.size();
    plan->view.buffers = plan->buffers.data();
    plan->view.n_buffers = (int64_t)plan->buffers.size();
    if (be->prepare_plan) {
        rc = be->prepare_plan(be->ctx, &plan->view);
        if (rc) {
            const std::string msg = fb::last_error();
            for (auto &b : plan->buffers) be->release_buffer(be->ctx, b.handle);
            return set_error(rc, "%s", msg.c_str());
        }
    }
    *out = plan.release();
    return FB_OK;
    GRAPH_END
}

const fb_plan *fb_plan_get(fb_compiled_plan *p) { return p ? &p->view : nullptr; }

int64_t fb_plan_find(fb_compiled_plan *p, uint32_t id) {
    if (!p) return -1;
    for (size_t i = 0; i < p->tensors.size(); i++)
        if (p->tensors[i].id == id) return (int64_t)i;
    return -1;
}

static uint64_t plan_tensor_nbytes(const fb_plan_tensor &t) {
    fb::Layout l;
    for (int i = 0; i < 4; i++) {
        l.shape.dims[i] = t.ne[i];
        l.stride[i] = t.nb[i];
    }
    return fb::layout_nbytes(l, t.dtype);
}

// plan.rs:77-95
int fb_plan_write_tensor(fb_compiled_plan *p, const fb_backend_vtable *be, uint32_t id, const void *src, uint64_t n) {
    if (!p || !be) return set_error(FB_ERR_INVALID, "write_tensor: null plan or backend");
    const int64_t i = fb_plan_find(p, id);
    if (i < 0) return set_error(FB_ERR_INVALID, "write_tensor: unknown tensor %u", id);
    const fb_plan_tensor &t = p->tensors[(size_t)i];
    const uint64_t nb = plan_tensor_nbytes(t);
    if (n != nb)
        return set_error(FB_ERR_SHAPE, "shape error: write_tensor: tensor %u needs %lu bytes, got %lu", id,
                         (unsigned long)nb, (unsigned long)n);
    return be->write(be->ctx, p->buffers[(size_t)t.buffer].handle, t.offset, src, n);
}

// plan.rs:97-115
int fb_plan_read_tensor(fb_compiled_plan *p, const fb_backend_vtable *be, uint32_t id, void *dst, uint64_t n) {
    if (!p || !be) return set_error(FB_ERR_INVALID, "read_tensor: null plan or backend");
    const int64_t i = fb_plan_find(p, id);
    if (i < 0) return set_error(FB_ERR_INVALID, "read_tensor: unknown tensor %u", id);
    const fb_plan_tensor &t = p->tensors[(size_t)i];
    const uint64_t nb = plan_tensor_nbytes(t);
    if (n != nb)
        return set_error(FB_ERR_SHAPE, "shape error: read_tensor: tensor %u needs %lu bytes, got %lu", id,
                         (unsigned long)nb, (unsigned long)n);
    return be->read(be->ctx, p->buffers[(size_t)t.buffer].handle, t.offset, dst, n);
}

// plan.rs:68-73
int fb_plan_release(fb_compiled_plan *p, const fb_backend_vtable *be) {
    if (!p || !be) return set_error(FB_ERR_INVALID, "release: null plan or backend");
    for (auto &b : p->buffers) {
        int rc = be->release_buffer(be->ctx, b.handle);
        if (rc) return rc;
    }
    p->released = true;
    return FB_OK;
}

void fb_plan_free(fb_compiled_plan *p) { delete p; }

int fb_planner_plan(const fb_planner_tensor *tensors, int64_t n, const int64_t *order, int64_t n_order,
                    int32_t *kinds, uint64_t *offsets, uint64_t *weights_size, uint64_t *compute_size) {
    if (!tensors || n < 0 || (!order && n_order > 0)) return set_error(FB_ERR_INVALID, "planner: bad arguments");
    try {
        std::vector<TensorMeta> ts;
        for (int64_t i = 0; i < n; i++) {
            const fb_planner_tensor &pt = tensors[i];
            Shape s;
            int rc = make_shape(pt.ne, pt.rank, &s);
            if (rc) return rc;
            TensorMeta m;
            rc = make_layout(pt.dtype, s, &m.layout);
            if (rc) return rc;
            m.id = pt.id;
            m.dtype = pt.dtype;
            m.flags = pt.flags;
            m.op = pt.op;
            for (int j = 0; j < pt.n_srcs && j < FB_MAX_SRC; j++) m.srcs.push_back(pt.srcs[j]);
            m.view_src = pt.view_src;
            m.layout.offset = pt.view_offset;
            ts.push_back(std::move(m));
        }
        std::vector<size_t> ord;
        for (int64_t i = 0; i < n_order; i++) {
            if (order[i] < 0 || order[i] >= n) return set_error(FB_ERR_INVALID, "planner: order index out of range");
            ord.push_back((size_t)order[i]);
        }
        Planner pl(ts);
        PlannerOutput po;
        int rc = pl.run(ord, &po);
        if (rc) return rc;
        for (int64_t i = 0; i < n; i++) {
            auto it = po.assignments.find(ts[(size_t)i].id);
            kinds[i] = it == po.assignments.end() ? -1 : it->second.kind;
            offsets[i] = it == po.assignments.end() ? 0 : it->second.offset;
        }
        if (weights_size) *weights_size = po.weights_size;
        if (compute_size) *compute_size = po.compute_size;
        return FB_OK;
    } catch (const std::exception &e) {
        return set_error(FB_ERR_INVALID, "host exception: %s", e.what());
    }
}

int fb_layout_new(int32_t dtype, const int64_t *dims, int32_t rank, uint64_t *nb) {
    Shape s;
    int rc = make_shape(dims, rank, &s);
    if (rc) return rc;
    fb::Layout l;
    rc = make_layout(dtype, s, &l);
    if (rc) return rc;
    for (int i = 0; i < 4; i++) nb[i] = l.stride[i];
    return FB_OK;
}

int fb_layout_nbytes(int32_t dtype, const int64_t *ne, const uint64_t *nb, uint64_t *nbytes) {
    if (!dtype_traits(dtype)) return set_error(FB_ERR_INVALID, "unknown dtype %d", dtype);
    fb::Layout l;
    for (int i = 0; i < 4; i++) {
        l.shape.dims[i] = ne[i];
        l.stride[i] = nb[i];
    }
    *nbytes = fb::layout_nbytes(l, dtype);
    return FB_OK;
}

int fb_dtype_traits(int32_t dtype, int64_t *block_size, int64_t *type_size, int32_t *quantized) {
    const DTypeTraits *t = dtype_traits(dtype);
    if (!t) return set_error(FB_ERR_INVALID, "unknown dtype %d", dtype);
    if (block_size) *block_size = t->block_size;
    if (type_size) *type_size = t->type_size;
    if (quantized) *quantized = t->quantized ? 1 : 0;
    return FB_OK;
}

}  // extern "C"
