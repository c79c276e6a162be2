"""Plan graphs: graph_compute replays a CUDA graph of a plan's launches from
its second call on (the reference's plan-caching hook is GraphPlan.uid,
feml-core/src/plan.rs:38-39). Replayed results equal node-by-node results
bit for bit, new inputs written between calls are seen, a plan recompiled
into new buffers (same uid) gets its own graph, and replays allocate
nothing."""
import numpy as np
import pytest

import feml_b200 as F
from feml_b200 import DType, GraphBuilder
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu
K, M = 4096, 256


def _decode_plan(be, rng):
    """x -> rms_norm -> (q: Q4_K, k: Q8_0) plus an unfused F32 projection and
    a 16-column Q4_0 GEMM on a second input: four kinds of launches."""
    g = GraphBuilder()
    wq = g.weight("wq", DType.Q4_K, [K, M])
    wk = g.weight("wk", DType.Q8_0, [K, M])
    wf = g.weight("wf", DType.F32, [512, 64])
    wg = g.weight("wg", DType.Q4_0, [K, M])
    x = g.input("x", DType.F32, [K, 1])
    xf = g.input("xf", DType.F32, [512, 4])
    xg = g.input("xg", DType.F32, [K, 16])
    r = g.rms_norm(x, 1e-5)
    q, k = g.mul_mat(wq, r), g.mul_mat(wk, r)
    f, h = g.mul_mat(wf, xf), g.mul_mat(wg, xg)
    for o in (q, k, f, h):
        g.mark_output(o)
    plan = g.compile(be)
    w = lambda m, k_: (rng.standard_normal((m, k_)) * 0.02).astype(np.float32)  # noqa: E731
    data = {"wq": O.quantize(O.DT_Q4_K, w(M, K)), "wk": O.quantize(O.DT_Q8_0, w(M, K)), "wf": w(64, 512),
            "wg": O.quantize(O.DT_Q4_0, w(M, K))}
    ids = {"wq": wq, "wk": wk, "wf": wf, "wg": wg, "x": x, "xf": xf, "xg": xg}
    for name in ("wq", "wk", "wf", "wg"):
        plan.write_tensor(be, ids[name], data[name])
    outs = {"q": (q, (1, M)), "k": (k, (1, M)), "f": (f, (4, 64)), "h": (h, (16, M))}
    return plan, ids, outs, data


def _step(be, plan, ids, outs, inputs):
    for name, arr in inputs.items():
        plan.write_tensor(be, ids[name], arr)
    be.graph_compute(plan)
    res = {}
    for name, (tid, shape) in outs.items():
        res[name] = np.empty(shape, np.float32)
        plan.read_tensor(be, tid, res[name])
    return res


def _inputs(rng):
    return {"x": rng.standard_normal((1, K)).astype(np.float32),
            "xf": rng.standard_normal((4, 512)).astype(np.float32),
            "xg": rng.standard_normal((16, K)).astype(np.float32)}


def test_replayed_plan_equals_node_by_node():
    graphs = F.B200Backend.open(0)
    eager = F.B200Backend.open(0)
    eager.set_plan_graphs(False)
    try:
        pg, ids_g, outs_g, data = _decode_plan(graphs, np.random.default_rng(1))
        pe, ids_e, outs_e, _ = _decode_plan(eager, np.random.default_rng(1))
        rng = np.random.default_rng(2)
        for step in range(4):
            inp = _inputs(rng)
            a = _step(graphs, pg, ids_g, outs_g, inp)
            b = _step(eager, pe, ids_e, outs_e, inp)
            for name in a:
                assert np.array_equal(a[name].view(np.uint32), b[name].view(np.uint32)), (step, name)
            if step == 0:
                before = graphs.device_allocations()
        assert graphs.plan_graphs() == (1, 1)
        assert eager.plan_graphs() == (0, 0)
        assert graphs.device_allocations() == before
        # the replayed results are the right ones
        x = inp["x"].astype(np.float64)
        xn = (inp["x"] * (1.0 / np.sqrt((x * x).mean() + 1e-5)).astype(np.float32)).astype(np.float32)
        ok, err = tol_ok(a["q"], O.mul_mat_quant_ref(O.DT_Q4_K, data["wq"], xn, K))
        assert ok, err
        ok, err = tol_ok(a["h"], O.mul_mat_quant_ref(O.DT_Q4_0, data["wg"], inp["xg"], K))
        assert ok, err
        assert np.array_equal(a["f"].view(np.uint32), O.mul_mat_f32(data["wf"], inp["xf"]).view(np.uint32))
        pg.release(graphs)
        pe.release(eager)
    finally:
        graphs.close()
        eager.close()


def test_recompiled_plan_gets_its_own_graph(b200):
    """Same graph structure (same uid) in new buffers: the cached graph of
    the released plan is not replayed into freed memory."""
    for seed in (3, 4):
        rng = np.random.default_rng(seed)
        plan, ids, outs, data = _decode_plan(b200, rng)
        inp = _inputs(rng)
        for _ in range(2):
            res = _step(b200, plan, ids, outs, inp)
        assert b200.plan_graphs()[1] >= 1
        ok, err = tol_ok(res["k"], O.mul_mat_quant_ref(
            O.DT_Q8_0, data["wk"],
            (inp["x"] * (1.0 / np.sqrt((inp["x"].astype(np.float64) ** 2).mean() + 1e-5))).astype(np.float32), K))
        assert ok, err
        plan.release(b200)
        assert b200.plan_graphs() == (0, 0)  # releasing buffers drops the graphs


def test_mul_mat_id_plan_replays():
    E, Km, Mm, N, n_sel = 4, 1024, 320, 24, 2
    rng = np.random.default_rng(9)
    wq = np.stack([O.quantize(O.DT_Q8_0, (rng.standard_normal((Mm, Km)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    be = F.B200Backend.open(0)
    try:
        g = GraphBuilder()
        w = g.weight("w", DType.Q8_0, [Km, Mm, E])
        xi = g.input("x", DType.F32, [Km, N])
        ii = g.input("ids", DType.I32, [n_sel, N])
        o = g.mul_mat_id(w, xi, ii, n_sel)
        g.mark_output(o)
        plan = g.compile(be)
        plan.write_tensor(be, w, wq)
        for step in range(3):
            x = rng.standard_normal((N, Km)).astype(np.float32)
            ids = np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)
            plan.write_tensor(be, xi, x)
            plan.write_tensor(be, ii, ids)
            be.graph_compute(plan)
            out = np.empty((N, n_sel, Mm), np.float32)
            plan.read_tensor(be, o, out)
            ok, err = tol_ok(out, O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, Km))
            assert ok, (step, err)
        assert be.plan_graphs() == (1, 1)
        plan.release(be)
    finally:
        be.close()
