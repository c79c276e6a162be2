"""GPU parity for mul_mat_id (ggml semantics: ids [n_selected, N], output
[M, n_selected, N]). Routing tables are bit-exact against the oracle's
stable order; outputs are within tolerance of the oracle's per-slot F32
mul_mat on dequantized operands; invalid ids give zero columns and an error
at synchronize (reported on the host, no device fault)."""
import numpy as np
import pytest
import torch

import feml_b200 as F
from feml_b200 import DType, ops
from oracle import oracle as O
from tests.conftest import tol_ok
from tests.gpu_helpers import run_mul_mat_id

pytestmark = pytest.mark.gpu
QT = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K, DType.F32: O.DT_F32}


def topk_ids(rng, N, n_sel, E):
    return np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)


@pytest.mark.parametrize("N,n_sel,E", [(1, 2, 8), (37, 2, 4), (512, 2, 8), (1500, 4, 64), (3000, 1, 256)])
def test_route_bit_exact(b200, N, n_sel, E):
    rng = np.random.default_rng(N + E)
    ids = topk_ids(rng, N, n_sel, E) if n_sel > 1 else rng.integers(0, E, (N, 1)).astype(np.int32)
    c, o, r = ops.moe_route(torch.from_numpy(ids).cuda(), E)
    torch.cuda.synchronize()
    wc, wo, wr, bad = O.moe_route(ids, E)
    assert bad == 0
    assert np.array_equal(c.cpu().numpy(), wc)
    assert np.array_equal(o.cpu().numpy(), wo)
    assert np.array_equal(r.cpu().numpy(), wr)


def _expert_weights(rng, dt, E, M, K):
    w = (rng.standard_normal((E, M, K)) * 0.02).astype(np.float32)
    if dt == DType.F32:
        return w
    return np.stack([O.quantize(QT[dt], w[e]) for e in range(E)])


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K, DType.F32])
@pytest.mark.parametrize("E,M,K,N,n_sel", [(4, 64, 256, 37, 2), (8, 200, 512, 5, 2), (3, 96, 1024, 130, 1),
                                           (8, 128, 256, 1, 2)])
def test_mul_mat_id_matches_oracle(b200, dt, E, M, K, N, n_sel):
    rng = np.random.default_rng(E * 100 + M + N)
    wb = _expert_weights(rng, dt, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = topk_ids(rng, N, n_sel, E)
    got = run_mul_mat_id(b200, dt, wb, x, ids, K, M)
    want = O.mul_mat_id_ref(QT[dt], wb, x, ids, K, quantize_act=dt != DType.F32)
    ok, err = tol_ok(got, want)
    assert ok, err


def test_mul_mat_id_bad_ids_zero_and_report(b200):
    rng = np.random.default_rng(1)
    E, M, K, N, n_sel = 4, 64, 256, 9, 2
    wb = _expert_weights(rng, DType.Q8_0, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = topk_ids(rng, N, n_sel, E)
    ids[3, 1] = 7
    ids[5, 0] = -1
    out, err = run_mul_mat_id(b200, DType.Q8_0, wb, x, ids, K, M, check_sync=False)
    assert isinstance(err, F.FemlError) and "out of range" in str(err)
    assert not out[3, 1].any() and not out[5, 0].any()
    want = O.mul_mat_id_ref(O.DT_Q8_0, wb, x, ids, K)
    ok, e = tol_ok(out, want)
    assert ok, e
    b200.synchronize()  # the status word was cleared: the backend stays usable


def test_mul_mat_id_equivalent_to_per_expert_mul_mat(b200):
    # the grouped kernel must give the same bits as mul_mat on each expert's
    # gathered columns when every column tile is full (192 columns; an
    # ungrouped product of at most 128 columns uses the stacked two-MMA form,
    # whose rounding differs)
    rng = np.random.default_rng(2)
    E, M, K, N = 2, 128, 512, 384
    wb = _expert_weights(rng, DType.Q8_0, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.zeros((N, 1), np.int32)
    ids[N // 2:] = 1
    got = run_mul_mat_id(b200, DType.Q8_0, wb, x, ids, K, M)
    wt = torch.from_numpy(wb).cuda()
    xt = torch.from_numpy(x).cuda()
    y0 = ops.mul_mat(DType.Q8_0, wt[0], xt[: N // 2], K).cpu().numpy()
    y1 = ops.mul_mat(DType.Q8_0, wt[1], xt[N // 2:], K).cpu().numpy()
    assert np.array_equal(got[: N // 2, 0], y0)
    assert np.array_equal(got[N // 2:, 0], y1)


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_K, DType.F32])
@pytest.mark.parametrize("n_shards", [2, 3, 8])
def test_mul_mat_id_shards_compose(b200, dt, n_shards):
    """Every shard writes only the slots of its own experts; the union over
    shards equals the unsharded mul_mat_id bit for bit (same per-output
    arithmetic) and the oracle within tolerance. Invalid ids are zeroed by
    every shard and reported."""
    rng = np.random.default_rng(40 + n_shards)
    E, M, K, N, n_sel = 5, 72, 512, 33, 2
    wb = _expert_weights(rng, dt, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = topk_ids(rng, N, n_sel, E)
    ids[3, 1] = -1
    wt = torch.from_numpy(np.ascontiguousarray(wb)).cuda()
    xt = torch.from_numpy(x).cuda()
    it = torch.from_numpy(ids).cuda()
    full = ops.mul_mat_id(dt, wt, xt, it, K)
    sentinel = torch.full((N, n_sel, M), float("nan"), device="cuda")
    union = torch.zeros_like(sentinel)
    for r in range(n_shards):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        part = sentinel.clone()
        ops.mul_mat_id_shard(dt, wt[r::n_shards], xt, it, K, E, r, n_shards, part, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) & 2, "invalid id not reported"
        mine = torch.from_numpy((ids % n_shards == r) & (ids >= 0) & (ids < E)).cuda()
        bad = torch.from_numpy((ids < 0) | (ids >= E)).cuda()
        assert torch.isnan(part[~(mine | bad)]).all(), "a shard wrote another shard's slot"
        assert (part[bad] == 0).all()
        union[mine] = part[mine]
    assert torch.equal(union, torch.nan_to_num(full.masked_fill(torch.from_numpy((ids < 0)[..., None]).cuda(), 0)))
    want = O.mul_mat_id_ref(QT[dt], wb, x, ids, K, quantize_act=dt != DType.F32)
    ok, err = tol_ok(union.cpu().numpy(), want)
    assert ok, err


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
def test_mul_mat_id_repeated_calls_are_deterministic(b200, dt):
    rng = np.random.default_rng(31)
    E, M, K, N, n_sel = 8, 1024, 2048, 400, 2
    wt = torch.from_numpy(np.ascontiguousarray(_expert_weights(rng, dt, E, M, K))).cuda()
    xt = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda()
    it = torch.from_numpy(topk_ids(rng, N, n_sel, E)).cuda()
    outs = [ops.mul_mat_id(dt, wt, xt, it, K) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0])
def test_mul_mat_id_expert_group_wider_than_a_tile(b200, dt):
    """One expert receives more routed slots than a column tile holds (the
    Q8_0 / Q4_0 GEMM's grouped tiles are 192 wide): its group spans a full
    tile and a narrow one; the weight rows end inside an m-tile."""
    rng = np.random.default_rng(41)
    E, M, K, N = 3, 200, 512, 260
    wb = _expert_weights(rng, dt, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.zeros((N, 1), np.int32)
    ids[230:245] = 1
    ids[245:] = 2
    got = run_mul_mat_id(b200, dt, wb, x, ids, K, M)
    want = O.mul_mat_id_ref(QT[dt], wb, x, ids, K, quantize_act=True)
    ok, err = tol_ok(got, want)
    assert ok, err


@pytest.mark.parametrize("dt,K", [(DType.Q8_0, 2048), (DType.Q4_0, 2048), (DType.Q4_K, 2048), (DType.Q4_K, 1280)])
def test_mul_mat_id_tail_split(b200, dt, K):
    """38 weight-row tiles x 4 expert column tiles = 152 tiles on 148 SMs:
    the grouped GEMM splits the last weight-row tile of every expert in K
    (planned in the kernel from the routed tile count) and a reduce kernel
    writes those outputs through the group map. M ends inside that tile.
    K = 1280 (Q4_K) runs the per-block kernel's 128-column tiles."""
    rng = np.random.default_rng(43)
    E, M, N, n_sel = 4, 4800, 100, 2
    wb = _expert_weights(rng, dt, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = topk_ids(rng, N, n_sel, E)
    got = run_mul_mat_id(b200, dt, wb, x, ids, K, M)
    want = O.mul_mat_id_ref(QT[dt], wb, x, ids, K, quantize_act=True)
    ok, err = tol_ok(got, want)
    assert ok, err
    wt = torch.from_numpy(wb).cuda()
    xt = torch.from_numpy(x).cuda()
    it = torch.from_numpy(ids).cuda()
    outs = [ops.mul_mat_id(dt, wt, xt, it, K) for _ in range(2)]
    assert torch.equal(outs[0], outs[1])
    assert np.array_equal(outs[0].cpu().numpy().reshape(got.shape), got)


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_K])
def test_mul_mat_id_long_rows_few_slots(b200, dt):
    """K = 8192 with 39 routed slots: the activation quantizer splits each
    slot's row over a cluster of CTAs; an invalid id leaves its slot out of
    the routed rows (those clusters return at once) and zero."""
    rng = np.random.default_rng(44)
    E, M, K, N, n_sel = 4, 256, 8192, 20, 2
    wb = _expert_weights(rng, dt, E, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = topk_ids(rng, N, n_sel, E)
    ids[7, 1] = E  # invalid: reported, its slot zero
    out, err = run_mul_mat_id(b200, dt, wb, x, ids, K, M, check_sync=False)
    assert isinstance(err, F.FemlError)
    assert not out[7, 1].any()
    want = O.mul_mat_id_ref(QT[dt], wb, x, ids, K, quantize_act=True)
    ok, e2 = tol_ok(out, want)
    assert ok, e2
    b200.synchronize()

