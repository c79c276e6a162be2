"""GPU parity at the full sizes of the benchmark workloads.

Every output of every workload (C1-C5) is compared with the oracle (the
multi-threaded C restatement of feml-cpu/src/ops/mul_mat.rs:36-57 on the
dequantized operands); C3 and C5 also check size-independent properties of
the whole output: power-of-two scaling of the activations scales every
output exactly, and permuting activation columns permutes output columns
exactly (each column's arithmetic is independent of its position). Weights
are drawn with numpy default_rng(seed) as in the workload definitions and
quantized by the oracle (bytes identical to the device quantizer, checked in
test_gpu_quant.py)."""
import numpy as np
import pytest
import torch

from feml_b200 import DType, ops
from oracle import oracle as O
from tests.conftest import tol_ok
from tests.gpu_helpers import run_mul_mat, run_mul_mat_id

pytestmark = pytest.mark.gpu


def test_c1_f32_4096x4096_n32(b200):
    rng = np.random.default_rng(0)
    K, M, N = 4096, 4096, 32
    w = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    x = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    got = run_mul_mat(b200, DType.F32, w, x, K, M)
    want = O.mul_mat_f32(w, x)
    ok, err = tol_ok(got, want)
    assert ok, err
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "not bit-exact"


def test_c2_q8_0_gemv_4096x4096(b200):
    rng = np.random.default_rng(1)
    K, M, N = 4096, 4096, 1
    wq = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    got = run_mul_mat(b200, DType.Q8_0, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q8_0, wq, x, K))
    assert ok, err


@pytest.mark.parametrize("N", [1, 8, 64])
def test_c4_q4_k_14336x4096(b200, N):
    rng = np.random.default_rng(3)
    K, M = 14336, 4096
    wq = O.quantize(O.DT_Q4_K, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    got = run_mul_mat(b200, DType.Q4_K, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
    assert ok, err


@pytest.fixture(scope="module")
def c3_data():
    rng = np.random.default_rng(2)
    K, M, N = 4096, 11008, 512
    wq = O.quantize(O.DT_Q4_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    return K, M, N, wq, x


def test_c3_q4_0_prefill_every_output(b200, c3_data):
    K, M, N, wq, x = c3_data
    got = run_mul_mat(b200, DType.Q4_0, wq, x, K, M)
    want = O.mul_mat_quant_ref(O.DT_Q4_0, wq, x, K)
    ok, err = tol_ok(got, want)
    assert ok, err


def test_c3_q4_0_prefill_properties(b200, c3_data):
    K, M, N, wq, x = c3_data
    wt = torch.from_numpy(wq).cuda()
    xt = torch.from_numpy(x).cuda()
    y = ops.mul_mat(DType.Q4_0, wt, xt, K)
    y8 = ops.mul_mat(DType.Q4_0, wt, xt * 8.0, K)
    perm = torch.from_numpy(np.random.default_rng(5).permutation(N)).cuda()
    yp = ops.mul_mat(DType.Q4_0, wt, xt[perm].contiguous(), K)
    torch.cuda.synchronize()
    assert torch.equal(y8, y * 8.0)
    assert torch.equal(yp, y[perm])


@pytest.fixture(scope="module")
def c5_data():
    rng = np.random.default_rng(4)
    E, M, K, N, n_sel = 8, 14336, 4096, 512, 2
    wq = np.stack([O.quantize(O.DT_Q8_0, rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02))
                   for _ in range(E)])
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)
    return E, M, K, N, n_sel, wq, x, ids


def test_c5_moe_q8_0_every_output(b200, c5_data):
    E, M, K, N, n_sel, wq, x, ids = c5_data
    got = run_mul_mat_id(b200, DType.Q8_0, wq, x, ids, K, M)
    want = O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, K)
    ok, err = tol_ok(got, want)
    assert ok, err


def test_c5_moe_q8_0_properties_and_routing(c5_data):
    E, M, K, N, n_sel, wq, x, ids = c5_data
    wt = torch.from_numpy(wq).cuda()
    xt, it = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    out = ops.mul_mat_id(DType.Q8_0, wt, xt, it, K)
    out2 = ops.mul_mat_id(DType.Q8_0, wt, xt * 2.0, it, K)
    perm = torch.from_numpy(np.random.default_rng(6).permutation(N)).cuda()
    outp = ops.mul_mat_id(DType.Q8_0, wt, xt[perm].contiguous(), it[perm].contiguous(), K)
    torch.cuda.synchronize()
    assert torch.equal(out2, out * 2.0)
    assert torch.equal(outp, out[perm])
    # routing at full size is bit-exact
    c, o, r = ops.moe_route(it, E)
    wc, wo, wr, bad = O.moe_route(ids, E)
    assert bad == 0 and np.array_equal(r.cpu().numpy(), wr) and np.array_equal(c.cpu().numpy(), wc)


def test_c5_through_graph_small_experts(b200):
    # the mul_mat_id node through compile/graph_compute at the workload's
    # K, token count and top-2 routing, with narrower experts
    rng = np.random.default_rng(4)
    E, M, K, N, n_sel = 8, 512, 4096, 512, 2
    w = (rng.standard_normal((E, M, K)) * 0.02).astype(np.float32)
    wq = np.stack([O.quantize(O.DT_Q8_0, w[e]) for e in range(E)])
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)
    got = run_mul_mat_id(b200, DType.Q8_0, wq, x, ids, K, M)
    ok, err = tol_ok(got, O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, K))
    assert ok, err
