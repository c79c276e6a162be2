"""mul_mat -> add(bias) -> silu fused into the mul_mat kernel's epilogue (the
compile-time fusion the reference plans, docs/DESIGN.md:250-251; ops
GraphBuilder::add / silu, feml-core/src/graph.rs:116-119,144-146).

Each case runs the chain twice through GraphBuilder -> compile ->
graph_compute: fused (intermediates are not outputs) and node by node (the
mul_mat output is marked as an output, which keeps the chain apart). The two
are bit-identical (same epilogue arithmetic), and both match the oracle:
F32 mul_mat on the dequantized operands (feml-cpu/src/ops/mul_mat.rs:36-57),
plus the bias (the reference's f32 add, feml-cpu/src/ops/elementwise.rs),
then SiLU, within the path's tolerance."""
import numpy as np
import pytest

from feml_b200 import DType, GraphBuilder
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu
CODE = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K, DType.F32: O.DT_F32}


def _run(be, dt, wb, x, bias, K, M, mode, keep_apart, bias_first=False):
    N = x.shape[0]
    g = GraphBuilder()
    wi = g.weight("w", dt, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    # a per-row bias is ne=[M, 1]: feml aligns broadcast dims from the last
    # one (feml-core/src/op.rs:116-136), so a rank-1 [M] would pair with N
    bi = g.input("b", DType.F32, [M, 1]) if bias is not None else None
    mm = g.mul_mat(wi, xi)
    t = mm
    if "bias" in mode:
        t = g.add(bi, t) if bias_first else g.add(t, bi)
    if "silu" in mode:
        t = g.silu(t)
    g.mark_output(t)
    if keep_apart:
        g.mark_output(mm)
    plan = g.compile(be)
    try:
        plan.write_tensor(be, wi, np.ascontiguousarray(wb))
        plan.write_tensor(be, xi, x)
        if bi is not None:
            plan.write_tensor(be, bi, bias)
        fused = be.plan_fused_nodes(plan)
        be.graph_compute(plan)
        be.synchronize()
        out = np.empty((N, M), np.float32)
        plan.read_tensor(be, t, out)
    finally:
        plan.release(be)
    return out, fused


CASES = [
    (DType.Q8_0, 4096, 1024, 1),    # decode GEMV, in-kernel activation quantization
    (DType.Q4_K, 14336, 512, 1),    # K-split GEMV
    (DType.Q4_K, 14336, 512, 8),    # K-split multi-column GEMV
    (DType.Q4_0, 4096, 1024, 256),  # tcgen05 GEMM with split-K (epilogue in the reduction)
    (DType.Q8_0, 4096, 2304, 200),  # tcgen05 GEMM, no split
    (DType.F32, 512, 256, 16),      # F32 mul_mat + a separate epilogue pass
]


@pytest.mark.parametrize("dt,K,M,N", CASES)
@pytest.mark.parametrize("mode", ["bias+silu", "bias", "silu"])
def test_fused_chain_equals_node_by_node_and_oracle(b200, dt, K, M, N, mode):
    rng = np.random.default_rng(K + M + N + len(mode))
    w = (rng.standard_normal((M, K)) * (0.02 if dt != DType.F32 else 0.05)).astype(np.float32)
    wb = w if dt == DType.F32 else O.quantize(CODE[dt], w)
    x = rng.standard_normal((N, K)).astype(np.float32)
    bias = (rng.standard_normal(M) * 0.5).astype(np.float32) if "bias" in mode else None
    got, n_fused = _run(b200, dt, wb, x, bias, K, M, mode, keep_apart=False)
    apart, n_apart = _run(b200, dt, wb, x, bias, K, M, mode, keep_apart=True)
    assert n_fused == mode.count("+") + 1 and n_apart == 0
    assert np.array_equal(got.view(np.uint32), apart.view(np.uint32)), "fused chain differs from node-by-node"
    want = O.mul_mat_quant_ref(CODE[dt], wb, x, K) if dt != DType.F32 else O.mul_mat_f32(w, x)
    if bias is not None:
        want = O.add_f32(want, bias[None, :])
    if "silu" in mode:
        want = O.silu_f32(want)
    ok, err = tol_ok(got, want)
    assert ok, err


def test_bias_as_first_add_operand_fuses_too(b200):
    rng = np.random.default_rng(5)
    # two columns: with one, the add's output is bias-sized and the planner
    # may place it in place over the bias input, which (correctly) keeps the
    # chain apart
    K, M, N = 4096, 512, 2
    wq = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    bias = rng.standard_normal(M).astype(np.float32)
    got, n = _run(b200, DType.Q8_0, wq, x, bias, K, M, "bias+silu", False, bias_first=True)
    apart, _ = _run(b200, DType.Q8_0, wq, x, bias, K, M, "bias+silu", True, bias_first=True)
    assert n == 2 and np.array_equal(got.view(np.uint32), apart.view(np.uint32))


def test_standalone_add_broadcasts_and_silu(b200):
    """The add and silu nodes on their own: ggml broadcasting ([4, 3] + [4, 1]
    and [1, 3] operands), exact f32 sums, SiLU to the oracle's f32 bits."""
    rng = np.random.default_rng(9)
    a = rng.standard_normal((3, 4)).astype(np.float32)   # ne = [4, 3]
    b = rng.standard_normal((1, 4)).astype(np.float32)   # ne = [4, 1]
    c = rng.standard_normal((3, 1)).astype(np.float32)   # ne = [1, 3]
    g = GraphBuilder()
    ai = g.input("a", DType.F32, [4, 3])
    bi = g.input("b", DType.F32, [4, 1])
    ci = g.input("c", DType.F32, [1, 3])
    s1 = g.add(ai, bi)
    s2 = g.add(s1, ci)
    y = g.silu(s2)
    g.mark_output(s2)
    g.mark_output(y)
    plan = g.compile(b200)
    try:
        plan.write_tensor(b200, ai, a)
        plan.write_tensor(b200, bi, b)
        plan.write_tensor(b200, ci, c)
        b200.graph_compute(plan)
        b200.synchronize()
        got_s = np.empty((3, 4), np.float32)
        got_y = np.empty((3, 4), np.float32)
        plan.read_tensor(b200, s2, got_s)
        plan.read_tensor(b200, y, got_y)
    finally:
        plan.release(b200)
    want_s = O.add_f32(O.add_f32(a, b), c)
    assert np.array_equal(got_s, want_s)
    assert np.max(np.abs(got_y - O.silu_f32(want_s))) <= 1e-6


def test_fused_chain_on_the_tail_split_gemm(b200):
    """The C3 shape (Q4_0 11008 x 4096 x 512: 344 tiles, more than two waves)
    runs its last tile rows split in K with a reduction kernel; the fused
    bias + SiLU epilogue lives in that reduction for those rows."""
    rng = np.random.default_rng(31)
    K, M, N = 4096, 11008, 512
    wq = O.quantize(O.DT_Q4_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    bias = (rng.standard_normal(M) * 0.5).astype(np.float32)
    got, n_fused = _run(b200, DType.Q4_0, wq, x, bias, K, M, "bias+silu", keep_apart=False)
    apart, _ = _run(b200, DType.Q4_0, wq, x, bias, K, M, "bias+silu", keep_apart=True)
    assert n_fused == 2
    assert np.array_equal(got.view(np.uint32), apart.view(np.uint32))
    want = O.silu_f32(O.add_f32(O.mul_mat_quant_ref(O.DT_Q4_0, wq, x, K), bias[None, :]))
    ok, err = tol_ok(got, want)
    assert ok, err
