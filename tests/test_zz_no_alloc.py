"""feml_b200_mul_mat_noalloc (the mul_mat whose scratch is the library's
fixed device array) against feml_b200_mul_mat with a caller workspace, both
through the C ABI. Both run the same kernels on the same inputs, so their
outputs must be identical bit for bit. Named to be collected last, so it
also runs after every other test in one process; it passes on its own in a
fresh process too."""
import numpy as np
import pytest
import torch

import feml_b200 as F
from feml_b200 import DType, ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu
QT = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}
SHAPES = [
    (DType.Q8_0, 4096, 4096, 8),    # quantized activations in scratch, GEMV on 8 columns
    (DType.Q4_0, 1024, 300, 33),    # tiled GEMM over the scratch activations
    (DType.Q4_K, 2048, 256, 1),     # fused GEMV: no scratch used
    (DType.Q8_0, 4096, 512, 400),   # large scratch (about 13 MB: operand planes + split-K partials)
]


def _two_calls_match(device, dt, K, M, N):
    with torch.cuda.device(device):
        rng = np.random.default_rng(K + M + N + 17 * device)
        wq = O.quantize(QT[dt], (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
        w = torch.from_numpy(wq).cuda(device)
        for call in range(2):  # two calls in a row share the scratch
            x = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda(device)
            want = ops.mul_mat(dt, w, x, K)
            got = torch.full((N, M), float("nan"), device=f"cuda:{device}")
            ops.mul_mat_noalloc(dt, w, x, K, got)
            torch.cuda.synchronize(device)
            assert torch.equal(got, want), (
                f"device {device} call {call}: max abs diff {(got - want).abs().max().item()}")


@pytest.mark.parametrize("dt,K,M,N", SHAPES)
def test_noalloc_matches_workspace_entry_point(dt, K, M, N):
    _two_calls_match(0, dt, K, M, N)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
@pytest.mark.parametrize("dt,K,M,N", [SHAPES[0], SHAPES[3]])
def test_noalloc_second_device_uses_its_own_array(dt, K, M, N):
    """Device 1 looks up its own copy of the array (no peer operands)."""
    _two_calls_match(1, dt, K, M, N)
    _two_calls_match(0, dt, K, M, N)


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    torch.cuda.set_device(0)
    limit = ops.mul_mat_noalloc_limit()
    K, M, N = 14336, 64, 1024
    assert ops.mul_mat_workspace(DType.Q4_K, K, M, N) > limit
    w = torch.zeros((M, DType.Q4_K.row_size(K)), dtype=torch.uint8, device="cuda")
    x = torch.zeros((N, K), dtype=torch.float32, device="cuda")
    out = torch.zeros((N, M), dtype=torch.float32, device="cuda")
    with pytest.raises(F.FemlError) as ei:
        ops.mul_mat_noalloc(DType.Q4_K, w, x, K, out)
    assert "static scratch" in str(ei.value)
    torch.cuda.synchronize()
    assert not out.any()


def test_noalloc_checks_arguments_before_the_size():
    """A negative dimension is an invalid argument (as for feml_b200_mul_mat),
    not a shape too large for the array; an empty output is a no-op; an
    unsupported weight dtype is rejected."""
    import ctypes
    from feml_b200 import _lib
    lib = _lib.lib()
    null = ctypes.c_void_p()
    invalid, unsupported = 1, 2  # FB_ERR_INVALID, FB_ERR_UNSUPPORTED (include/feml_b200.h)
    rc = lib.feml_b200_mul_mat_noalloc(int(DType.Q8_0), null, 0, null, 0, null, 0, 4096, 64, -1, null)
    assert rc == invalid
    assert "negative" in lib.feml_b200_last_error().decode()
    assert lib.feml_b200_mul_mat_noalloc(int(DType.Q8_0), null, 0, null, 0, null, 0, 4096, 0, 8, null) == 0
    rc = lib.feml_b200_mul_mat_noalloc(int(DType.I32), null, 0, null, 0, null, 0, 4096, 64, 8, null)
    assert rc == unsupported
