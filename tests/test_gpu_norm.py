"""rms_norm (Op::RmsNorm, feml-core/src/op.rs:26; GraphBuilder::rms_norm,
graph.rs:140-142) on the B200 backend: as its own node (materialized), and
fused into the decode GEMV's activation quantization when a plan feeds it
straight into mul_mat. Outputs within the path's tolerance of the oracle's
mul_mat on numpy-normalized activations."""
import numpy as np
import pytest

from feml_b200 import DType, GraphBuilder
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu
QT = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K, DType.Q5_K: O.DT_Q5_K}
EPS = 1e-5


def rms_norm_ref(x, eps=EPS):
    """Per row (ne0 contiguous): x / sqrt(mean(x^2) + eps), f32 result."""
    x64 = x.astype(np.float64)
    scale = (1.0 / np.sqrt((x64 * x64).mean(axis=-1, keepdims=True) + eps)).astype(np.float32)
    return (x * scale).astype(np.float32)


def _run(be, build, feeds, reads):
    g = GraphBuilder()
    ids = build(g)
    plan = g.compile(be)
    try:
        for name, arr in feeds.items():
            plan.write_tensor(be, ids[name], np.ascontiguousarray(arr))
        be.graph_compute(plan)
        be.synchronize()
        out = {}
        for name, shape in reads.items():
            out[name] = np.empty(shape, np.float32)
            plan.read_tensor(be, ids[name], out[name])
        return out
    finally:
        plan.release(be)


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K, DType.Q5_K])
@pytest.mark.parametrize("K,M,N", [(4096, 300, 1), (2048, 129, 3), (512, 64, 8), (14336, 200, 1)])
def test_rms_norm_fused_into_mul_mat(b200, dt, K, M, N):
    rng = np.random.default_rng(K + M + N + int(dt))
    wq = O.quantize(QT[dt], (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = (rng.standard_normal((N, K)) * 3.0 + 0.5).astype(np.float32)

    def build(g):
        w = g.weight("w", dt, [K, M])
        xi = g.input("x", DType.F32, [K, N])
        r = g.rms_norm(xi, EPS)
        y = g.mul_mat(w, r)
        g.mark_output(y)
        return {"w": w, "x": xi, "y": y}

    got = _run(b200, build, {"w": wq, "x": x}, {"y": (N, M)})["y"]
    ok, err = tol_ok(got, O.mul_mat_quant_ref(QT[dt], wq, rms_norm_ref(x), K))
    assert ok, err


def test_rms_norm_materialized_when_it_is_an_output(b200):
    """An rms_norm that is a graph output runs as its own kernel; its values
    and the mul_mat reading it both match."""
    K, M, N = 4096, 256, 2
    rng = np.random.default_rng(3)
    wq = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)

    def build(g):
        w = g.weight("w", DType.Q8_0, [K, M])
        xi = g.input("x", DType.F32, [K, N])
        r = g.rms_norm(xi, EPS)
        y = g.mul_mat(w, r)
        g.mark_output(r)
        g.mark_output(y)
        return {"w": w, "x": xi, "r": r, "y": y}

    out = _run(b200, build, {"w": wq, "x": x}, {"r": (N, K), "y": (N, M)})
    want_r = rms_norm_ref(x)
    assert np.allclose(out["r"], want_r, rtol=2e-6, atol=1e-7)
    ok, err = tol_ok(out["y"], O.mul_mat_quant_ref(O.DT_Q8_0, wq, want_r, K))
    assert ok, err


def test_rms_norm_feeding_two_projections(b200):
    """One normalized activation read by two decode mul_mats (q and k
    projections): both fused."""
    K, M, N = 4096, 192, 1
    rng = np.random.default_rng(4)
    wq = O.quantize(O.DT_Q4_K, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    wk = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)

    def build(g):
        a = g.weight("wq", DType.Q4_K, [K, M])
        b = g.weight("wk", DType.Q8_0, [K, M])
        xi = g.input("x", DType.F32, [K, N])
        r = g.rms_norm(xi, EPS)
        q = g.mul_mat(a, r)
        k = g.mul_mat(b, r)
        g.mark_output(q)
        g.mark_output(k)
        return {"wq": a, "wk": b, "x": xi, "q": q, "k": k}

    out = _run(b200, build, {"wq": wq, "wk": wk, "x": x}, {"q": (N, M), "k": (N, M)})
    xn = rms_norm_ref(x)
    for name, w, t in (("q", wq, O.DT_Q4_K), ("k", wk, O.DT_Q8_0)):
        ok, err = tol_ok(out[name], O.mul_mat_quant_ref(t, w, xn, K))
        assert ok, (name, err)


@pytest.mark.parametrize("dt", [DType.Q4_0, DType.F32])
def test_rms_norm_unfused_shapes(b200, dt):
    """Shapes outside the fused GEMV (64 columns: the tiled GEMM; F32
    weights) normalize in the rms_norm kernel first."""
    K, M, N = 1024, 160, 64
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    wb = w if dt == DType.F32 else O.quantize(O.DT_Q4_0, w)
    x = rng.standard_normal((N, K)).astype(np.float32)

    def build(g):
        wi = g.weight("w", dt, [K, M])
        xi = g.input("x", DType.F32, [K, N])
        y = g.mul_mat(wi, g.rms_norm(xi, EPS))
        g.mark_output(y)
        return {"w": wi, "x": xi, "y": y}

    got = _run(b200, build, {"w": wb, "x": x}, {"y": (N, M)})["y"]
    xn = rms_norm_ref(x)
    want = O.mul_mat_f32(w, xn) if dt == DType.F32 else O.mul_mat_quant_ref(O.DT_Q4_0, wb, xn, K)
    ok, err = tol_ok(got, want)
    assert ok, err


def test_rms_norm_rank3_standalone(b200):
    K = 96
    rng = np.random.default_rng(6)
    x = rng.standard_normal((3, 5, K)).astype(np.float32)

    def build(g):
        xi = g.input("x", DType.F32, [K, 5, 3])
        r = g.rms_norm(xi, 1e-6)
        g.mark_output(r)
        return {"x": xi, "r": r}

    out = _run(b200, build, {"x": x}, {"r": (3, 5, K)})["r"]
    assert np.allclose(out, rms_norm_ref(x, 1e-6), rtol=2e-6, atol=1e-7)
