"""The multi-GPU wrappers with their CUDA compute step, on a one-rank NCCL
group (the multi-rank collective logic is covered on gloo ranks in
test_shard.py; multi-GPU runs use bench.py --gpus N)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist

from feml_b200 import DType, ops
from feml_b200.shard import ExpertShardedMulMatId, RowShardedMulMat
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def group():
    if not dist.is_initialized():
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(0)
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", 0))
        yield None
        dist.destroy_process_group()
    else:
        yield None


@pytest.mark.parametrize("N", [1, 8, 64])
def test_row_sharded_q4_k(group, N):
    rng = np.random.default_rng(3 + N)
    K, M = 2048, 300
    wq = O.quantize(O.DT_Q4_K, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((N, K)).astype(np.float32)
    op = RowShardedMulMat(DType.Q4_K, torch.from_numpy(wq).cuda(), K, M)
    y = op(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    want = O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K)
    ok, err = tol_ok(y.cpu().numpy(), want)
    assert ok, err


def test_expert_sharded_q8_0(group):
    rng = np.random.default_rng(4)
    E, M, K, N, n_sel = 8, 96, 512, 40, 2
    wq = np.stack([O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)
    op = ExpertShardedMulMatId(DType.Q8_0, torch.from_numpy(wq).cuda(), K, E)
    out = op(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    want = O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, K)
    ok, err = tol_ok(out.cpu().numpy(), want)
    assert ok, err


def test_row_sharded_fused_single_rank(group):
    """The fused path (peer stores + flag + device-side epoch) on a one-rank
    group: the same kernel arithmetic as the unfused GEMV, over several steps
    (the output buffers alternate)."""
    rng = np.random.default_rng(7)
    K, M = 14336, 512
    wq = O.quantize(O.DT_Q4_K, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    wt = torch.from_numpy(wq).cuda()
    fused = RowShardedMulMat(DType.Q4_K, wt, K, M, fused=True)
    plain = RowShardedMulMat(DType.Q4_K, wt, K, M)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in range(3):
        x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).cuda()
        got = fused(x).clone()
        want = plain(x)
        torch.cuda.synchronize()
        assert torch.equal(got, want), step
        ok, err = tol_ok(got.cpu().numpy(), O.mul_mat_quant_ref(O.DT_Q4_K, wq, x.cpu().numpy(), K))
        assert ok, err
    assert int(status.item()) == 0


def test_expert_sharded_fused_single_rank(group):
    """The fused expert-sharded combine (grouped tcgen05 epilogue storing into
    the peer buffers) on a one-rank group: bitwise the unfused result over
    several steps, an invalid id giving a zero slot in both."""
    rng = np.random.default_rng(8)
    E, M, K, N, n_sel = 4, 300, 512, 40, 2
    wq = np.stack([O.quantize(O.DT_Q4_K, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    wt = torch.from_numpy(wq).cuda()
    fused = ExpertShardedMulMatId(DType.Q4_K, wt, K, E, fused=True, max_tokens=64, max_selected=4)
    plain = ExpertShardedMulMatId(DType.Q4_K, wt, K, E)
    for step in range(3):
        n = N - 7 * step  # ragged token counts reuse the same buffers
        x = torch.from_numpy(rng.standard_normal((n, K)).astype(np.float32)).cuda()
        ids_np = np.stack([rng.permutation(E)[:n_sel] for _ in range(n)]).astype(np.int32)
        ids_np[3, 1] = E  # invalid id: zero slot
        ids = torch.from_numpy(ids_np).cuda()
        got = fused(x, ids).clone()
        want = plain(x, ids)
        torch.cuda.synchronize()
        assert torch.equal(got, want), step
        assert not got[3, 1].any()
    fused.close()
    ok, err = tol_ok(got.cpu().numpy(), O.mul_mat_id_ref(O.DT_Q4_K, wq, x.cpu().numpy(), ids_np, K))
    assert ok, err


def test_expert_sharded_fused_owner_single_rank(group):
    """The owner combine (each slot stored only into the buffer of the rank
    owning its token) on a one-rank group owns every token: bitwise the
    unfused result over ragged steps, an invalid id giving a zero slot."""
    rng = np.random.default_rng(9)
    E, M, K, N, n_sel = 4, 260, 512, 40, 2
    wq = np.stack([O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    wt = torch.from_numpy(wq).cuda()
    fused = ExpertShardedMulMatId(DType.Q8_0, wt, K, E, fused=True, max_tokens=64, max_selected=4, combine="owner")
    plain = ExpertShardedMulMatId(DType.Q8_0, wt, K, E)
    for step in range(3):
        n = N - 9 * step
        x = torch.from_numpy(rng.standard_normal((n, K)).astype(np.float32)).cuda()
        ids_np = np.stack([rng.permutation(E)[:n_sel] for _ in range(n)]).astype(np.int32)
        ids_np[2, 0] = -1  # invalid id: zero slot
        ids = torch.from_numpy(ids_np).cuda()
        assert fused.token_range(n) == (0, n)
        got = fused(x, ids).clone()
        want = plain(x, ids)
        torch.cuda.synchronize()
        assert torch.equal(got, want), step
        assert not got[2, 0].any()
    fused.close()


def _fused_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    rng = np.random.default_rng(11)
    K, M = 8192, 1000
    wq = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    wt = torch.from_numpy(wq).cuda()
    fused = RowShardedMulMat(DType.Q8_0, wt, K, M, fused=True)
    worst = 0.0
    for step in range(4):
        x = torch.from_numpy(rng.standard_normal((2, K)).astype(np.float32)).cuda()
        got = fused(x).clone()
        want = ops.mul_mat(DType.Q8_0, wt, x, K)
        torch.cuda.synchronize()
        worst = max(worst, float((got - want).abs().max()))
    fused.close()
    np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([worst]))
    dist.barrier()
    dist.destroy_process_group()


def _fused_id_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    rng = np.random.default_rng(12)
    E, M, K, N, n_sel = 8, 200, 1024, 70, 2
    wq = np.stack([O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    wt = torch.from_numpy(wq).cuda()
    fused = ExpertShardedMulMatId(DType.Q8_0, wt, K, E, fused=True, max_tokens=N, max_selected=n_sel)
    worst = 0.0
    for step in range(4):
        x = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda()
        ids = torch.from_numpy(np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)).cuda()
        got = fused(x, ids).clone()
        want = ops.mul_mat_id(DType.Q8_0, wt, x, ids, K)
        torch.cuda.synchronize()
        worst = max(worst, float((got - want).abs().max()))
    fused.close()
    np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([worst]))
    dist.barrier()
    dist.destroy_process_group()


def _fused_id_owner_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    rng = np.random.default_rng(13)
    E, M, K, N, n_sel = 8, 200, 1024, 70, 2
    wq = np.stack([O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
                   for _ in range(E)])
    wt = torch.from_numpy(wq).cuda()
    fused = ExpertShardedMulMatId(DType.Q8_0, wt, K, E, fused=True, max_tokens=N, max_selected=n_sel,
                                  combine="owner")
    worst = 0.0
    for step in range(4):
        n = N - 5 * step
        x = torch.from_numpy(rng.standard_normal((n, K)).astype(np.float32)).cuda()
        ids = torch.from_numpy(np.stack([rng.permutation(E)[:n_sel] for _ in range(n)]).astype(np.int32)).cuda()
        lo, hi = fused.token_range(n)
        got = fused(x, ids).clone()
        want = ops.mul_mat_id(DType.Q8_0, wt, x, ids, K)[lo:hi]
        torch.cuda.synchronize()
        worst = max(worst, float((got - want).abs().max()) if hi > lo else 0.0)
    fused.close()
    np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([worst]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_fused_worker, _fused_id_worker, _fused_id_owner_worker],
                         ids=["rows", "experts", "experts-owner"])
def test_sharded_fused_two_gpus(tmp_path, worker):
    """Peer stores over NVLink between two processes (needs two GPUs): the
    gathered rows / combined expert slots equal the one-GPU result bitwise."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert float(np.load(tmp_path / f"r{r}.npy")[0]) == 0.0
