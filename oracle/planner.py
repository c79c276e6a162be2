"""Memory planner restated in Python -- TEST INFRASTRUCTURE ONLY.

Follows feml-core/src/planner.rs step for step (the ggml-alloc algorithm the
reference ports): `Talloc` first-fit over an unsorted free list whose split
remainders are appended, sort + coalesce on free, 32-byte alignment
(planner.rs:53-99); `can_reuse` (:105-115); `allocate` with lazy view
resolution (:129-152); `plan` (:156-261): INPUT / WEIGHT leaves first in
tensor order, then every node in topological order with in-place reuse of a
sole parent and freeing at the last use. Used by tests/test_planner_fuzz.py
to check the product planner (feml_b200/csrc/graph.cpp) on random graphs.

Tensors are dicts: id, nbytes, flags, op, srcs (ids, duplicates allowed),
view_src (id or None), view_offset, dtype, shape (for the reuse rule).
"""

ALIGNMENT = 32
INPUT, OUTPUT, WEIGHT = 1, 2, 4
# op.rs:98-110 (Op discriminants as in feml-core/src/op.rs:12-43)
NONE, VIEW, MUL, ADD, MUL_MAT, MUL_MAT_ID, RMS_NORM, SOFTMAX, ROPE, SILU, GET_ROWS, CONCAT, COPY, DIAG_MASK_INF, \
    SCALE = range(15)
INPLACE = {MUL, ADD, RMS_NORM, SILU, SOFTMAX, ROPE, DIAG_MASK_INF, SCALE}
WEIGHTS, COMPUTE = 0, 1


def _round(v):
    return (v + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


class Talloc:
    def __init__(self):
        self.used = 0
        self.free_list = []

    def alloc(self, size):
        size = _round(size)
        for idx, (off, fsize) in enumerate(self.free_list):
            if fsize >= size:
                del self.free_list[idx]
                if fsize > size:
                    self.free_list.append((off + size, fsize - size))
                return off
        off = _round(self.used)
        self.used = off + size
        return off

    def free(self, off, size):
        self.free_list.append((off, _round(size)))
        self.free_list.sort()
        merged = []
        for o, s in self.free_list:
            if merged and merged[-1][0] + merged[-1][1] == o:
                merged[-1] = (merged[-1][0], merged[-1][1] + s)
            else:
                merged.append((o, s))
        self.free_list = merged


def _kind(t):
    return WEIGHTS if t["flags"] & WEIGHT else COMPUTE


def _can_reuse(node, parent, children, views):
    return (node["op"] in INPLACE and children == 1 and views == 0 and not parent["flags"] & OUTPUT
            and not parent["flags"] & WEIGHT and node["dtype"] == parent["dtype"]
            and list(node["shape"]) == list(parent["shape"]))


def plan(tensors, order):
    """-> ({id: (kind, offset)}, weights_size, compute_size)"""
    by_id = {t["id"]: t for t in tensors}
    children = {t["id"]: 0 for t in tensors}
    views = {t["id"]: 0 for t in tensors}
    for t in tensors:
        if t.get("view_src") is not None:
            views[t["view_src"]] += 1
        for s in t["srcs"]:
            children[s] += 1
    talloc = [Talloc(), Talloc()]
    assigned, allocated = {}, {t["id"]: False for t in tensors}
    live_children, live_views = dict(children), dict(views)

    def allocate(tid):
        if allocated[tid]:
            return
        t = by_id[tid]
        if t.get("view_src") is not None:
            allocate(t["view_src"])
            kind, off = assigned[t["view_src"]]
            assigned[tid] = (kind, off + t["view_offset"])
            allocated[tid] = True
            return
        k = _kind(t)
        assigned[tid] = (k, talloc[k].alloc(t["nbytes"]))
        allocated[tid] = True

    for t in tensors:
        if t["flags"] & (INPUT | WEIGHT):
            allocate(t["id"])

    for idx in order:
        node = tensors[idx]
        nid = node["id"]
        if node.get("view_src") is not None:
            allocate(node["view_src"])
            kind, off = assigned[node["view_src"]]
            assigned[nid] = (kind, off + node["view_offset"])
            allocated[nid] = True
        else:
            for s in node["srcs"]:
                if not allocated[s]:
                    allocate(s)
            reused = False
            if node["op"] in INPLACE:
                for s in node["srcs"]:
                    parent = by_id[s]
                    if (allocated[s] and live_children[s] == 1 and live_views[s] == 0
                            and _can_reuse(node, parent, live_children[s], live_views[s])):
                        assigned[nid] = assigned[s]
                        allocated[nid] = True
                        allocated[s] = False
                        reused = True
                        break
            if not reused:
                k = _kind(node)
                assigned[nid] = (k, talloc[k].alloc(node["nbytes"]))
                allocated[nid] = True
        for s in node["srcs"]:
            live_children[s] -= 1
            parent = by_id[s]
            never_freed = parent["flags"] & (INPUT | WEIGHT | OUTPUT)
            if live_children[s] == 0 and live_views[s] == 0 and not never_freed:
                if allocated[s]:
                    kind, off = assigned[s]
                    talloc[kind].free(off, parent["nbytes"])
                    allocated[s] = False
                elif parent.get("view_src") is not None:
                    vs = parent["view_src"]
                    live_views[vs] -= 1
                    if (live_views[vs] == 0 and live_children[vs] == 0 and not by_id[vs]["flags"] & OUTPUT
                            and allocated[vs]):
                        kind, off = assigned[vs]
                        talloc[kind].free(off, by_id[vs]["nbytes"])
                        allocated[vs] = False
    return assigned, talloc[WEIGHTS].used, talloc[COMPUTE].used
