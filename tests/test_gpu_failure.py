"""Failure detection on the GPU without a fault: the device-side wait that
ends a fused multi-GPU step (feml_b200_peer_wait_timeout) is given a flag that
nothing raises. It must give up within its bound, report STATUS_TIMEOUT in the
caller's status word, leave the epoch unchanged and leave the context usable.
The reference reports failures only as host-side error returns
(feml-cpu/tests/cpu_integration.rs:131-144); a lost rank is detected here the
same way, as an error status the host reads."""
import time

import numpy as np
import pytest
import torch

from feml_b200 import DType, ops
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu
STATUS_TIMEOUT = 1


def _mul_mat_still_right():
    rng = np.random.default_rng(7)
    K, M = 1024, 256
    wq = O.quantize(O.DT_Q8_0, (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((1, K)).astype(np.float32)
    y = ops.mul_mat(DType.Q8_0, torch.from_numpy(wq).cuda(), torch.from_numpy(x).cuda(), K)
    torch.cuda.synchronize()
    ok, err = tol_ok(y.cpu().numpy(), O.mul_mat_quant_ref(O.DT_Q8_0, wq, x, K))
    assert ok, err


@pytest.mark.parametrize("timeout_us", [2000, 50000])
def test_peer_wait_on_a_flag_nobody_raises_times_out(timeout_us):
    torch.cuda.set_device(0)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ops.peer_wait(flag, epoch, 2, status=status, timeout_us=timeout_us)  # a peer that never signals
    torch.cuda.synchronize()  # returns: the wait ended on its bound
    elapsed = time.perf_counter() - t0
    assert status.item() & STATUS_TIMEOUT
    assert epoch.item() == 0
    assert elapsed >= timeout_us * 1e-6 * 0.9
    assert elapsed < 5.0
    _mul_mat_still_right()
    # the same wait with every rank's signal present completes and advances the epoch
    flag.fill_(2)
    status.zero_()
    ops.peer_wait(flag, epoch, 2, status=status, timeout_us=timeout_us)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert epoch.item() == 1


def test_peer_wait_default_bound_ends():
    """The default wait (feml_b200_peer_wait) is bounded too (about a second)."""
    torch.cuda.set_device(0)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    ops.peer_wait(flag, epoch, 1, status=status)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert status.item() & STATUS_TIMEOUT
    _mul_mat_still_right()


def test_peer_wait_rejects_unbounded_timeouts():
    from feml_b200 import FemlError
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    for bad in (0, 10_000_001):
        with pytest.raises(FemlError):
            ops.peer_wait(flag, epoch, 1, timeout_us=bad)
