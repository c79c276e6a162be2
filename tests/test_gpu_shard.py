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
