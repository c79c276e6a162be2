"""Multi-rank logic of feml_b200.shard on gloo ranks (CPU, no GPU).

The compute step is the oracle here (injected), so these tests check the
sharding, the collectives and the reassembly: a sharded run must give the
same bytes as the single-device oracle. The CUDA compute step of the same
wrappers is covered by the GPU tests.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_mul_mat(wtype, w_local, x, K, out):
    y = O.mul_mat_quant_ref(int(wtype), w_local.numpy(), x.numpy(), K, nthreads=1)
    out.copy_(torch.from_numpy(y))


def _oracle_mul_mat_id(wtype, w_local, x, ids, K, n_experts, shard, n_shards, out):
    ids_np = ids.numpy()
    xs = x.numpy()
    for t in range(ids_np.shape[0]):
        for s in range(ids_np.shape[1]):
            e = int(ids_np[t, s])
            if 0 <= e < n_experts and e % n_shards == shard:
                y = O.mul_mat_quant_ref(int(wtype), w_local[e // n_shards].numpy(), xs[t:t + 1], K, nthreads=1)
                out[t, s].copy_(torch.from_numpy(y[0]))


def _row_case(seed, wtype, K, M, N):
    rng = np.random.default_rng(seed)
    wq = O.quantize(wtype, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    x = rng.normal(0, 1, (N, K)).astype(np.float32)
    return wq, x


def _expert_case(seed, wtype, K, M, E, N, n_sel, bad_id):
    rng = np.random.default_rng(seed)
    wq = np.stack([O.quantize(wtype, rng.normal(0, 0.02, (M, K)).astype(np.float32)) for _ in range(E)])
    x = rng.normal(0, 1, (N, K)).astype(np.float32)
    ids = np.stack([rng.choice(E, n_sel, replace=False) for _ in range(N)]).astype(np.int32)
    if bad_id:
        ids[N // 2, 0] = E + 3
    return wq, x, ids


def _row_worker(rank, world, port, case, outdir):
    from feml_b200.shard import RowShardedMulMat
    _init(rank, world, port)
    wtype, K, M, N, seed = case
    wq, x = _row_case(seed, wtype, K, M, N)
    op = RowShardedMulMat(wtype, torch.from_numpy(wq), K, M, compute=_oracle_mul_mat)
    y = op(torch.from_numpy(x))
    np.save(os.path.join(outdir, f"y{rank}.npy"), y.numpy())
    dist.destroy_process_group()


def _expert_worker(rank, world, port, case, outdir, combine="replicate"):
    from feml_b200.shard import ExpertShardedMulMatId
    _init(rank, world, port)
    wtype, K, M, E, N, n_sel, bad, seed = case
    wq, x, ids = _expert_case(seed, wtype, K, M, E, N, n_sel, bad)
    op = ExpertShardedMulMatId(wtype, torch.from_numpy(wq), K, E, compute_id=_oracle_mul_mat_id, max_tokens=N,
                               combine=combine)
    out = op(torch.from_numpy(x), torch.from_numpy(ids))
    np.save(os.path.join(outdir, f"y{rank}.npy"), out.numpy())
    np.save(os.path.join(outdir, f"range{rank}.npy"), np.array(op.token_range(N) if combine == "owner" else (0, N)))
    dist.destroy_process_group()


def _missing_rank_worker(rank, world, port, outdir):
    """Rank 1 never joins the gather; rank 0's collective must end in an
    error within the process-group timeout instead of waiting for good."""
    import time
    from feml_b200.shard import RowShardedMulMat
    _init(rank, world, port, timeout_s=3)
    wq, x = _row_case(9, O.DT_Q8_0, 64, 8, 1)
    if rank == 1:
        time.sleep(6)
        open(os.path.join(outdir, "r1"), "w").write("skipped")
        return
    op = RowShardedMulMat(O.DT_Q8_0, torch.from_numpy(wq), 64, 8, compute=_oracle_mul_mat)
    t0 = time.time()
    try:
        op(torch.from_numpy(x))
        msg = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        msg = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"
    open(os.path.join(outdir, "r0"), "w").write(msg)


def _spawn(fn, world, *args):
    mp.start_processes(fn, args=(world, _free_port()) + args, nprocs=world, join=True, start_method="spawn")


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("wtype,K,M,N", [(O.DT_Q4_K, 512, 37, 1), (O.DT_Q8_0, 128, 20, 5), (O.DT_Q4_0, 64, 9, 3),
                                      (O.DT_Q5_K, 256, 11, 2), (O.DT_Q6_K, 256, 13, 1)])
def test_row_shard_matches_single_device(tmp_path, world, wtype, K, M, N):
    case = (wtype, K, M, N, 3)
    _spawn(_row_worker, world, case, str(tmp_path))
    wq, x = _row_case(3, wtype, K, M, N)
    want = O.mul_mat_quant_ref(wtype, wq, x, K, nthreads=1)
    for r in range(world):
        got = np.load(tmp_path / f"y{r}.npy")
        assert got.shape == (N, M)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {r}"


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("bad", [False, True])
def test_expert_shard_matches_single_device(tmp_path, world, bad):
    case = (O.DT_Q8_0, 64, 12, 5, 7, 2, bad, 4)
    _spawn(_expert_worker, world, case, str(tmp_path))
    wq, x, ids = _expert_case(4, O.DT_Q8_0, 64, 12, 5, 7, 2, bad)
    want = O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, 64, nthreads=1)
    for r in range(world):
        got = np.load(tmp_path / f"y{r}.npy")
        assert got.shape == want.shape
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {r}"


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("bad", [False, True])
def test_expert_shard_owner_combine(tmp_path, world, bad):
    """combine="owner": each rank ends with exactly its own tokens' slots
    (token t on rank t // ceil(N / world)); together they are the
    single-device result, every token once."""
    N = 7
    case = (O.DT_Q8_0, 64, 12, 5, N, 2, bad, 5)
    _spawn(_expert_worker, world, case, str(tmp_path), "owner")
    wq, x, ids = _expert_case(5, O.DT_Q8_0, 64, 12, 5, N, 2, bad)
    want = O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, 64, nthreads=1)
    covered = []
    T = -(-N // world)
    for r in range(world):
        lo, hi = np.load(tmp_path / f"range{r}.npy")
        assert (lo, hi) == (min(N, r * T), min(N, r * T + T))
        got = np.load(tmp_path / f"y{r}.npy")
        assert got.shape == (hi - lo,) + want.shape[1:]
        assert np.array_equal(got.view(np.uint32), want[lo:hi].view(np.uint32)), f"rank {r}"
        covered += list(range(lo, hi))
    assert covered == list(range(N))


def test_rank_that_skips_the_gather_times_out(tmp_path):
    _spawn(_missing_rank_worker, 2, str(tmp_path))
    msg = (tmp_path / "r0").read_text()
    assert msg.startswith("error"), msg
    assert float(msg.split()[2].rstrip("s:")) < 30


def test_row_ranges_cover_rows_once():
    from feml_b200.shard import row_range, local_experts
    for M in (1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                lo, hi, R = row_range(M, r, world)
                assert 0 <= hi - lo <= R
                seen += list(range(lo, hi))
            assert seen == list(range(M))
    for E in (1, 5, 8):
        for world in (1, 2, 3, 8):
            assert sum(local_experts(E, r, world) for r in range(world)) == E
