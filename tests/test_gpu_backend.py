"""GPU: the Backend contract through the C ABI, mirroring the reference's
CUDA integration tests (feml-cuda/tests/cuda_integration.rs) and the backend
test requirements (docs/backend-guide.md:98-103): buffer lifecycle, one
numeric op against the known answers, cross-checking with the CPU path."""
import json
import os

import numpy as np
import pytest

import feml_b200 as F
from feml_b200 import BufferUsage, DType, FemlError, GraphBuilder, Op
from oracle import oracle as O
from tests.conftest import tol_ok
from tests.gpu_helpers import run_mul_mat

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_registrar_reports_devices():
    reg = F.B200Registrar.probe()
    assert reg.name() == "B200"
    assert reg.device_count() >= 1 and reg.score() > 1000
    info = reg.device(0).info()
    assert info["compute_capability"] == (10, 0) and info["sm_count"] > 0 and info["memory_total"] > 0


def test_registry_open_best_picks_b200():
    r = F.Registry().register(F.B200Registrar.probe())
    be = r.open_best()
    assert be.name() == "B200"
    be.close()


def test_fill_and_read_roundtrip(b200):
    buf = b200.create_buffer(64, BufferUsage.COMPUTE)
    b200.fill(buf, 0, 0xAB, 64)
    b200.synchronize()
    assert bytes(b200.read(buf, 0, 64)) == b"\xab" * 64
    b200.release_buffer(buf)


def test_create_buffer_is_zeroed(b200):
    buf = b200.create_buffer(4097, BufferUsage.WEIGHTS)
    assert bytes(b200.read(buf, 0, 4097)) == bytes(4097)
    b200.release_buffer(buf)


def test_write_read_partial_offset(b200):
    buf = b200.create_buffer(16, BufferUsage.COMPUTE)
    b200.fill(buf, 0, 0, 16)
    b200.write(buf, 8, bytes([1, 2, 3]))
    out = bytes(b200.read(buf, 0, 16))
    assert out == bytes(8) + bytes([1, 2, 3]) + bytes(5)
    b200.release_buffer(buf)


def test_out_of_bounds_rejected(b200):
    buf = b200.create_buffer(8, BufferUsage.COMPUTE)
    with pytest.raises(FemlError):
        b200.write(buf, 4, bytes([1, 2, 3, 4, 5]))
    with pytest.raises(FemlError):
        b200.read(buf, 4, 5)
    with pytest.raises(FemlError):
        b200.fill(buf, 7, 0, 2)
    with pytest.raises(FemlError):
        b200.write(buf, 2 ** 64 - 4, bytes(8))  # offset + n overflows
    b200.release_buffer(buf)


def test_unknown_handle_rejected(b200):
    with pytest.raises(FemlError):
        b200.read(999999, 0, 1)
    with pytest.raises(FemlError):
        b200.release_buffer(999999)


def _ramp(name):
    with open(os.path.join(GOLD, "mul_mat_ramp.json")) as f:
        c = json.load(f)[name]
    K, M, N = c["K"], c["M"], c["N"]
    w = np.array(c["w_bits"], dtype=np.uint32).view(np.float32).reshape(M, K)
    x = np.array(c["x_bits"], dtype=np.uint32).view(np.float32).reshape(N, K)
    want = np.array(c["want_bits"], dtype=np.uint32).view(np.float32).reshape(N, M)
    return w, x, want, K, M


def test_mul_mat_matches_reference(b200):
    # feml-cuda/tests/cuda_integration.rs:211-244, tolerance 1e-3
    w, x, want, K, M = _ramp("cpu_integration_mul_mat_matches_reference")
    got = run_mul_mat(b200, DType.F32, w, x, K, M)
    assert np.max(np.abs(got - want)) < 1e-3


def test_cpu_and_b200_agree(b200):
    # feml-cuda/tests/cuda_integration.rs:246-278 against the CPU restatement
    w, x, want, K, M = _ramp("cuda_integration_cpu_and_cuda_agree")
    cpu = O.mul_mat_f32(w, x)
    got = run_mul_mat(b200, DType.F32, w, x, K, M)
    assert np.max(np.abs(got - cpu)) < 1e-3


def test_plan_release_frees_buffers(b200):
    g = GraphBuilder()
    w = g.weight("w", DType.F32, [16, 8])
    x = g.input("x", DType.F32, [16, 4])
    o = g.mul_mat(w, x)
    g.mark_output(o)
    plan = g.compile(b200)
    handle = plan.buffers[plan.find(o).buffer].handle
    plan.release(b200)
    with pytest.raises(FemlError):
        b200.read(handle, 0, 4)


def test_unsupported_op_rejected_at_compile(b200):
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    g.mark_output(g.mul(a, b))
    with pytest.raises(FemlError) as e:
        g.compile(b200)
    assert "does not support op mul" in str(e.value)


def test_graph_compute_is_async_until_synchronize(b200):
    rng = np.random.default_rng(11)
    K, M, N = 4096, 512, 1
    w = rng.standard_normal((M, K)).astype(np.float32) * 0.02
    wq = O.quantize(O.DT_Q8_0, w)
    x = rng.standard_normal((N, K)).astype(np.float32)
    g = GraphBuilder()
    wi = g.weight("w", DType.Q8_0, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    o = g.mul_mat(wi, xi)
    g.mark_output(o)
    plan = g.compile(b200)
    plan.write_tensor(b200, wi, wq)
    plan.write_tensor(b200, xi, x)
    for _ in range(50):  # repeated execution of one plan reuses everything
        b200.graph_compute(plan)
    b200.synchronize()
    out = np.empty((N, M), np.float32)
    plan.read_tensor(b200, o, out)
    plan.release(b200)
    ok, err = tol_ok(out, O.mul_mat_quant_ref(O.DT_Q8_0, wq, x, K))
    assert ok, err


def test_mul_mat_rejects_aliasing_dst(b200):
    # a hand-built plan whose dst overlaps its weights must be rejected
    g = GraphBuilder()
    w = g.weight("w", DType.F32, [16, 8])
    x = g.input("x", DType.F32, [16, 4])
    o = g.mul_mat(w, x)
    g.mark_output(o)
    plan = g.compile(b200)
    p = plan._plan_ptr().contents
    idx = [i for i in range(p.n_tensors) if p.tensors[i].id == o][0]
    src = [i for i in range(p.n_tensors) if p.tensors[i].id == x][0]
    p.tensors[idx].buffer = p.tensors[src].buffer
    p.tensors[idx].offset = p.tensors[src].offset
    with pytest.raises(FemlError) as e:
        b200.graph_compute(plan)
    assert "aliases" in str(e.value)
    plan.release(b200)


@pytest.mark.parametrize("dt,K,M,N", [(DType.Q8_0, 4096, 512, 1), (DType.Q4_0, 4096, 1024, 64),
                                      (DType.Q4_K, 14336, 256, 8), (DType.F32, 512, 64, 32)])
def test_second_graph_compute_allocates_nothing(b200, dt, K, M, N):
    """The zero-allocation contract of graph_compute (docs/backend-guide.md:22,
    checked in feml-cpu/tests/cpu_integration.rs:230-251 with a counting
    allocator): after a plan's first graph_compute, further calls make no
    device allocation."""
    rng = np.random.default_rng(K + N)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    wb = w if dt == DType.F32 else O.quantize({DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0,
                                                DType.Q4_K: O.DT_Q4_K}[dt], w)
    g = GraphBuilder()
    wi = g.weight("w", dt, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    o = g.mul_mat(wi, xi)
    g.mark_output(o)
    plan = g.compile(b200)
    try:
        plan.write_tensor(b200, wi, wb)
        plan.write_tensor(b200, xi, rng.standard_normal((N, K)).astype(np.float32))
        b200.graph_compute(plan)
        b200.synchronize()
        first = np.empty((N, M), np.float32)
        plan.read_tensor(b200, o, first)
        before = b200.device_allocations()
        for _ in range(3):
            b200.graph_compute(plan)
        b200.synchronize()
        assert b200.device_allocations() == before
        again = np.empty((N, M), np.float32)
        plan.read_tensor(b200, o, again)
        assert np.array_equal(first, again)
    finally:
        plan.release(b200)


@pytest.mark.parametrize("dt,K,M,N", [(DType.Q4_K, 14336, 4096, 64), (DType.Q4_0, 4096, 1024, 64),
                                      (DType.Q8_0, 4096, 512, 1)])
def test_first_graph_compute_allocates_nothing(b200, dt, K, M, N):
    """compile prepares the plan (feml_b200_prepare_plan through the vtable):
    the scratch is sized for its largest node (split-K partials included) and
    its launches are captured, so even the first graph_compute allocates
    nothing (docs/backend-guide.md:22) and replays a graph."""
    code = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}[dt]
    rng = np.random.default_rng(K + M + N)
    wb = O.quantize(code, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    g = GraphBuilder()
    wi = g.weight("w", dt, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    o = g.mul_mat(wi, xi)
    g.mark_output(o)
    plan = g.compile(b200)
    try:
        before = b200.device_allocations()
        cached, replayable = b200.plan_graphs()
        assert replayable >= 1
        plan.write_tensor(b200, wi, wb)
        plan.write_tensor(b200, xi, x)
        b200.graph_compute(plan)
        b200.synchronize()
        assert b200.device_allocations() == before
        assert b200.plan_graphs() == (cached, replayable)
        got = np.empty((N, M), np.float32)
        plan.read_tensor(b200, o, got)
        ok, err = tol_ok(got, O.mul_mat_quant_ref(code, wb, x, K))
        assert ok, err
    finally:
        plan.release(b200)
