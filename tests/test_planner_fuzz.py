"""The product planner (feml_b200/csrc/graph.cpp, reached through
fb_planner_plan) against oracle/planner.py, a step-for-step Python
restatement of feml-core/src/planner.rs, on random graphs: inputs and
weights (F32 and Q8_0), in-place unary and binary ops, non-in-place ops,
views at aligned offsets, outputs. Every tensor's (buffer, offset) and both
buffer sizes must agree exactly: plans built by the reference's planner and
by this library address the same bytes. No GPU needed."""
import numpy as np
import pytest

import feml_b200 as F
from feml_b200 import DType, Op, TensorFlags
from oracle import planner as P

IN, OUT, W = TensorFlags.INPUT, TensorFlags.OUTPUT, TensorFlags.WEIGHT


def _nbytes(dtype, shape):
    n = DType(dtype).row_size(shape[0])
    for d in shape[1:]:
        n *= d
    return n


def _random_graph(rng):
    shapes = [[64], [64, 2], [32, 4], [128], [256, 3]]
    tensors = []

    def add(shape, flags=0, op=Op.NONE, srcs=(), view_src=0, view_offset=0, dtype=DType.F32):
        t = {"id": len(tensors) + 1, "shape": list(shape), "flags": flags, "op": op, "srcs": list(srcs),
             "view_src": view_src, "view_offset": view_offset, "dtype": dtype}
        tensors.append(t)
        return t

    for _ in range(int(rng.integers(2, 5))):
        add(shapes[int(rng.integers(len(shapes)))], IN)
    if rng.random() < 0.7:
        add([64, 8], W, dtype=DType.Q8_0)
    n_leaves = len(tensors)
    for _ in range(int(rng.integers(3, 12))):
        f32 = [t for t in tensors if t["dtype"] == DType.F32]
        kind = rng.random()
        flags = OUT if rng.random() < 0.2 else 0
        a = f32[int(rng.integers(len(f32)))]
        if kind < 0.3:  # in-place unary
            add(a["shape"], flags, [Op.SILU, Op.RMS_NORM, Op.SCALE][int(rng.integers(3))], [a["id"]])
        elif kind < 0.55:  # in-place binary on equal shapes (sometimes the same source twice)
            same = [t for t in f32 if t["shape"] == a["shape"]]
            b = same[int(rng.integers(len(same)))]
            add(a["shape"], flags, [Op.ADD, Op.MUL][int(rng.integers(2))], [a["id"], b["id"]])
        elif kind < 0.7:  # not in place
            add(a["shape"], flags, Op.COPY, [a["id"]])
        elif kind < 0.85 and any(t["dtype"] == DType.Q8_0 for t in tensors):
            w = next(t for t in tensors if t["dtype"] == DType.Q8_0)
            xs = [t for t in f32 if t["shape"][0] == 64]
            if xs:
                x = xs[int(rng.integers(len(xs)))]
                n = x["shape"][1] if len(x["shape"]) > 1 else 1
                add([8, n], flags, Op.MUL_MAT, [w["id"], x["id"]])
        else:  # view at a 32-byte-aligned offset, then a reader of the view
            nb = _nbytes(a["dtype"], a["shape"])
            if nb >= 64:
                ve = int(rng.integers(1, nb // 4 // 2 + 1))
                off = int(rng.integers(0, (nb - 4 * ve) // 32 + 1)) * 32
                v = add([ve], 0, Op.VIEW, [], view_src=a["id"], view_offset=off)
                add([ve], flags, Op.SILU if rng.random() < 0.5 else Op.COPY, [v["id"]])
    order = list(range(n_leaves, len(tensors)))
    return tensors, order


@pytest.mark.parametrize("seed", range(300))
def test_planner_matches_reference_restatement(seed):
    rng = np.random.default_rng(seed)
    tensors, order = _random_graph(rng)
    got, ws, cs = F.planner_plan(tensors, order)
    ref_in = [{"id": t["id"], "nbytes": _nbytes(t["dtype"], t["shape"]), "flags": int(t["flags"]),
               "op": int(t["op"]), "srcs": t["srcs"], "view_src": t["view_src"] or None,
               "view_offset": t["view_offset"], "dtype": int(t["dtype"]), "shape": t["shape"]} for t in tensors]
    want, wws, wcs = P.plan(ref_in, order)
    assert (ws, cs) == (wws, wcs)
    for tid, (kind, off) in want.items():
        assert got[tid] == (kind, off), (tid, got[tid], (kind, off))


def test_restatement_reproduces_the_reference_known_answers():
    """The restatement itself, on the reference's planner tests
    (planner.rs:284-398): diamond 64, in-place 32, reuse of a freed slot 128."""
    def t(i, shape, flags=0, op=P.NONE, srcs=()):
        return {"id": i, "nbytes": 4 * int(np.prod(shape)), "flags": flags, "op": op, "srcs": list(srcs),
                "view_src": None, "view_offset": 0, "dtype": 5, "shape": shape}
    _, _, cs = P.plan([t(1, [4], P.INPUT), t(2, [4], P.INPUT), t(3, [4], 0, P.MUL, [1, 2]),
                       t(4, [4], 0, P.MUL, [1, 3])], [2, 3])
    assert cs == 64
    _, _, cs = P.plan([t(1, [8], P.INPUT), t(2, [8], 0, P.SILU, [1])], [1])
    assert cs == 32
    _, _, cs = P.plan([t(1, [16], P.INPUT), t(2, [16], P.INPUT), t(3, [16], 0, P.MUL, [1, 2]),
                       t(4, [16], 0, P.MUL, [3, 2])], [2, 3])
    assert cs == 128
