"""feml_b200_mul_mat_noalloc (the mul_mat whose scratch is the library's
fixed device array) against feml_b200_mul_mat with a caller workspace, both
through the C ABI. Named to be collected last, so it also runs after every
other test in one process; it passes on its own in a fresh process too."""
import numpy as np
import pytest
import torch

import feml_b200 as F
from feml_b200 import DType, ops
from oracle import oracle as O
from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu
QT = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}


@pytest.mark.parametrize("dt,K,M,N", [
    (DType.Q8_0, 4096, 4096, 8),    # quantized activations in scratch, GEMV on 8 columns
    (DType.Q4_0, 1024, 300, 33),    # tiled GEMM over the scratch activations
    (DType.Q4_K, 2048, 256, 1),     # fused GEMV: no scratch used
    (DType.Q8_0, 4096, 512, 600),   # large scratch (about 9.8 MB)
])
def test_noalloc_matches_workspace_entry_point(dt, K, M, N):
    torch.cuda.set_device(0)
    rng = np.random.default_rng(K + M + N)
    wq = O.quantize(QT[dt], (rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    w = torch.from_numpy(wq).cuda()
    for call in range(2):  # two calls in a row share the scratch
        x = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda()
        want = ops.mul_mat(dt, w, x, K)
        got = torch.full((N, M), float("nan"), device="cuda")
        ops.mul_mat_noalloc(dt, w, x, K, got)
        torch.cuda.synchronize()
        ok, err = tol_ok(got.cpu().numpy(), want.cpu().numpy())
        assert ok, f"call {call}: max abs diff {err}"


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
