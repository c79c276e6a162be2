"""GPU parity for the quantized mul_mat path.

Bit-exact: the device quantizers (quantize_row_q8_0 on activations, the
Q8_0/Q4_0/Q4_K weight quantizers) and the per-block int32 sums.
Within tolerance (|got - want| <= 1e-3 + 1e-4*|want|): mul_mat outputs
against the oracle's F32 mul_mat on the identically dequantized weights and
dequantized Q8_0 activations (the reference has no quant kernel, so its F32
mul_mat on dequantized operands is the parity target)."""
import os

import numpy as np
import pytest
import torch

import feml_b200 as F
from feml_b200 import DType
from feml_b200 import ops
from oracle import oracle as O
from tests.conftest import tol_ok
from tests.gpu_helpers import run_mul_mat, weights

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
QT = {DType.Q8_0: O.DT_Q8_0, DType.Q4_0: O.DT_Q4_0, DType.Q4_K: O.DT_Q4_K}


def _inputs(seed, rows, k):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x[0, :32] = 0.0                       # zero block
    x[0, 32:64] = -0.0
    x[1 % rows, :32] = np.arange(32, dtype=np.float32) - 15.5   # exact .5 products
    if rows > 2:
        x[2, :32] = 7.0                   # constant block
        x[2, 64:96] = np.where(np.arange(32) % 2 == 0, 3.0, -3.0)
    return x


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
def test_device_quantizer_bit_exact_golden(b200, dt):
    gv = np.load(os.path.join(GOLD, "quant_vectors.npz"))
    x = torch.from_numpy(gv["x"]).cuda()
    got = ops.quantize(dt, x).cpu().numpy()
    assert np.array_equal(got, gv[dt.name.lower()])


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
@pytest.mark.parametrize("rows,k,scale", [(7, 256, 1.0), (64, 4096, 0.02), (3, 14336, 3.0), (33, 768, 1e-3)])
def test_device_quantizer_bit_exact_random(b200, dt, rows, k, scale):
    x = _inputs(rows * 1000 + k, rows, k) * np.float32(scale)
    got = ops.quantize(dt, torch.from_numpy(x).cuda()).cpu().numpy()
    want = O.quantize(QT[dt], x)
    assert np.array_equal(got, want)


def test_quantize_row_q8_0_activations_bit_exact(b200):
    # the activation quantizer at the decode shape, with a strided source
    x = _inputs(5, 16, 4096)
    xt = torch.from_numpy(np.pad(x, ((0, 0), (0, 64)))).cuda()[:, :4096]
    got = ops.quantize(DType.Q8_0, xt).cpu().numpy()
    assert np.array_equal(got, O.quantize(O.DT_Q8_0, x))


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
@pytest.mark.parametrize("K,M,N", [(256, 5, 1), (1024, 33, 3), (4096, 64, 2)])
def test_block_dots_bit_exact(b200, dt, K, M, N):
    rng = np.random.default_rng(K + M + N)
    w = weights(rng, M, K, std=0.5)
    x = _inputs(K, N, K)
    wq = O.quantize(QT[dt], w)
    xq = O.quantize(O.DT_Q8_0, x)
    want, _ = O.block_dots(QT[dt], wq, xq, M, K, N)
    got = ops.block_dots(dt, torch.from_numpy(wq).cuda(), torch.from_numpy(xq).cuda(), K).cpu().numpy()
    assert np.array_equal(got, want)


SHAPES = [
    (256, 7, 1), (512, 33, 2), (1024, 130, 3), (4096, 256, 4),     # decode GEMV, fused quantization
    (512, 100, 5), (1024, 64, 8), (2048, 70, 7),                    # ... five to eight columns
    (8192, 40, 4), (4096, 300, 6),                                  # GEMV with a pre-quantized activation buffer
    (256, 300, 16), (2048, 200, 64),                                # GEMM path
    (768, 150, 33), (256, 1, 100), (4096, 257, 128), (512, 130, 300),
    (8192, 70, 20), (14336, 40, 9),                                 # long rows: cluster-split activation quantizer
]


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
@pytest.mark.parametrize("K,M,N", SHAPES)
def test_mul_mat_quant_matches_oracle(b200, dt, K, M, N):
    rng = np.random.default_rng(K * 7 + M * 3 + N)
    w = weights(rng, M, K)
    x = _inputs(K + N, N, K)
    wq = O.quantize(QT[dt], w)
    got = run_mul_mat(b200, dt, wq, x, K, M)
    want = O.mul_mat_quant_ref(QT[dt], wq, x, K)
    ok, err = tol_ok(got, want)
    assert ok, f"max abs err {err}"


@pytest.mark.parametrize("K,M", [(12288, 1000), (13056, 300), (14336, 5), (14336, 1), (16384, 37), (14336, 3584)])
def test_q4_k_wide_rows_one_column(b200, K, M):
    """Wide Q4_K rows at one column: the K-split GEMV (each warp one slice of
    K for all its CTA's rows, activations quantized per lane into registers,
    slices added in warp order). Ragged slices (13056 = 51 super-blocks),
    tiny M, repeated calls bit-identical."""
    rng = np.random.default_rng(K + 5 * M)
    w = weights(rng, M, K)
    x = _inputs(K + 1, 1, K)
    wq = O.quantize(O.DT_Q4_K, w)
    got = run_mul_mat(b200, DType.Q4_K, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
    assert ok, f"max abs err {err}"
    wt = torch.from_numpy(wq).cuda()
    xt = torch.from_numpy(x).cuda()
    outs = [ops.mul_mat(DType.Q4_K, wt, xt, K) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert np.array_equal(outs[0].cpu().numpy(), got)


@pytest.mark.parametrize("K,M,N", [(14336, 4096, 8), (12288, 1000, 2), (13056, 300, 5), (14336, 9, 7),
                                   (16384, 37, 3), (14336, 1, 8), (14336, 3584, 6)])
def test_q4_k_wide_rows_few_columns(b200, K, M, N):
    """Wide Q4_K rows at 2..8 columns: the K-split GEMV over planar
    activations (weight words of a box held in registers, columns walked per
    box, transposing warp reduction). Ragged slices (13056 = 51
    super-blocks), tiny M, repeated calls bit-identical."""
    rng = np.random.default_rng(K + 7 * M + N)
    wq = O.quantize(O.DT_Q4_K, weights(rng, M, K))
    x = _inputs(K + N, N, K)
    got = run_mul_mat(b200, DType.Q4_K, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
    assert ok, f"max abs err {err}"
    wt = torch.from_numpy(wq).cuda()
    xt = torch.from_numpy(x).cuda()
    outs = [ops.mul_mat(DType.Q4_K, wt, xt, K) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert np.array_equal(outs[0].cpu().numpy(), got)


def test_q4_k_wide_rows_few_columns_padded_stride(b200):
    """Weight rows and output columns with strides wider than their rows."""
    K, M, N = 14336, 700, 4
    rng = np.random.default_rng(98)
    wq = O.quantize(O.DT_Q4_K, weights(rng, M, K))
    rb = wq.shape[1]
    buf = torch.full((M, rb + 48), 0xAB, dtype=torch.uint8, device="cuda")
    buf[:, :rb] = torch.from_numpy(wq).cuda()
    x = _inputs(4, N, K)
    out = torch.full((N, M + 5), float("nan"), device="cuda")
    ops.mul_mat(DType.Q4_K, buf[:, :rb], torch.from_numpy(x).cuda(), K, out=out[:, :M])
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ok, err = tol_ok(got[:, :M], O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
    assert ok, err
    assert np.isnan(got[:, M:]).all()


@pytest.mark.parametrize("K,M,N", [(256, 7, 1), (4096, 300, 1), (14336, 64, 1), (768, 130, 3), (4096, 100, 8),
                                   (2048, 70, 12), (512, 33, 33), (11008, 40, 2)])
def test_mul_mat_q6_k_matches_oracle(b200, K, M, N):
    """Q6_K weights (210-byte super-blocks, 2-byte aligned: rows of K = 768
    or 11008 are not 16-byte multiples, so chunks carry ragged head and tail
    bytes) on the decode GEMV; layout pinned to gguf-py's dequantizer."""
    rng = np.random.default_rng(K + 5 * M + N)
    wq = O.quantize(O.DT_Q6_K, weights(rng, M, K))
    x = _inputs(K + 3 * N, N, K)
    got = run_mul_mat(b200, DType.Q6_K, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q6_K, wq, x, K))
    assert ok, f"max abs err {err}"
    wt, xt = torch.from_numpy(wq).cuda(), torch.from_numpy(x).cuda()
    a, b = ops.mul_mat(DType.Q6_K, wt, xt, K), ops.mul_mat(DType.Q6_K, wt, xt, K)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and np.array_equal(a.cpu().numpy(), got)


@pytest.mark.parametrize("K,M,N", [(256, 7, 1), (4096, 300, 1), (14336, 64, 1), (1024, 130, 3), (4096, 100, 8),
                                   (2048, 70, 12), (512, 33, 33)])
def test_mul_mat_q5_k_matches_oracle(b200, K, M, N):
    """Q5_K weights (block format pinned to gguf-py's dequantizer) through
    the graph path: the decode GEMV for N <= 8 (fused or planar activation
    quantization), column groups of eight beyond."""
    rng = np.random.default_rng(K + 3 * M + N)
    wq = O.quantize(O.DT_Q5_K, weights(rng, M, K))
    x = _inputs(K + 2 * N, N, K)
    got = run_mul_mat(b200, DType.Q5_K, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q5_K, wq, x, K))
    assert ok, f"max abs err {err}"
    wt, xt = torch.from_numpy(wq).cuda(), torch.from_numpy(x).cuda()
    a, b = ops.mul_mat(DType.Q5_K, wt, xt, K), ops.mul_mat(DType.Q5_K, wt, xt, K)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and np.array_equal(a.cpu().numpy(), got)


def test_q4_k_wide_rows_padded_stride(b200):
    """Row stride larger than the row (16-byte multiple): the 2D tensor map
    walks rows by the stride, not the row size."""
    K, M = 14336, 700
    rng = np.random.default_rng(99)
    wq = O.quantize(O.DT_Q4_K, weights(rng, M, K))
    rb = wq.shape[1]
    buf = torch.full((M, rb + 48), 0xAB, dtype=torch.uint8, device="cuda")
    buf[:, :rb] = torch.from_numpy(wq).cuda()
    x = _inputs(3, 1, K)
    got = ops.mul_mat(DType.Q4_K, buf[:, :rb], torch.from_numpy(x).cuda(), K)
    torch.cuda.synchronize()
    ok, err = tol_ok(got.cpu().numpy(), O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
    assert ok, err


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0])
@pytest.mark.parametrize("K,M,N", [(96, 40, 1), (160, 9, 6), (32, 3, 2), (288, 70, 12)])
def test_mul_mat_ragged_k(b200, dt, K, M, N):
    # K not a multiple of 256: row bytes not 16-aligned, TMA interior + plain edges
    rng = np.random.default_rng(K + N)
    w = weights(rng, M, K, std=1.0)
    x = _inputs(K, N, K)
    wq = O.quantize(QT[dt], w)
    got = run_mul_mat(b200, dt, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(QT[dt], wq, x, K))
    assert ok, err


@pytest.mark.parametrize("K,M,N", [
    (16, 8, 32), (4096, 64, 32), (100, 37, 5), (1000, 129, 1), (64, 3, 70),  # pipelined kernel
    (4100, 70, 33), (132, 1, 1), (256, 4001, 3),    # a 4-wide last k chunk, one row, many row tiles
    (99, 37, 5), (6, 9, 40),                        # K % 4 != 0: the cp.async kernel
])
def test_mul_mat_f32_matches_oracle(b200, K, M, N):
    """F32 mul_mat equals the reference CPU kernel's sequential f32 sums bit
    for bit (the reference's own CUDA kernel is built with fmad=false for the
    same reason)."""
    rng = np.random.default_rng(K + M + N)
    w = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    x = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    got = run_mul_mat(b200, DType.F32, w, x, K, M)
    want = O.mul_mat_f32(w, x)
    ok, err = tol_ok(got, want)
    assert ok, err
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "not bit-exact"


def test_mul_mat_f32_strided_operands(b200):
    """Row strides wider than the rows (16-byte multiples and not) on the
    kernel-level entry point; outputs bit-exact."""
    rng = np.random.default_rng(7)
    K, M, N = 520, 150, 9
    w = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    x = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    want = O.mul_mat_f32(w, x)
    for pad in (4, 1):
        wb = torch.zeros((M, K + pad), dtype=torch.float32, device="cuda")
        xb = torch.zeros((N, K + pad), dtype=torch.float32, device="cuda")
        wb[:, :K] = torch.from_numpy(w).cuda()
        xb[:, :K] = torch.from_numpy(x).cuda()
        got = ops.mul_mat(DType.F32, wb[:, :K], xb[:, :K], K)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32)), pad


def test_kernel_level_entry_matches_graph_path(b200):
    rng = np.random.default_rng(3)
    K, M, N = 4096, 300, 6
    w = weights(rng, M, K)
    x = rng.standard_normal((N, K)).astype(np.float32)
    wq = O.quantize(O.DT_Q4_0, w)
    via_graph = run_mul_mat(b200, DType.Q4_0, wq, x, K, M)
    via_ops = ops.mul_mat(DType.Q4_0, torch.from_numpy(wq).cuda(), torch.from_numpy(x).cuda(), K)
    torch.cuda.synchronize()
    assert np.array_equal(via_ops.cpu().numpy(), via_graph)


def test_scaling_by_power_of_two_is_exact(b200):
    # size-independent property: x -> 4x scales every Q8_0 scale by 4 exactly
    # and leaves the integers unchanged, so y scales exactly
    rng = np.random.default_rng(9)
    K, M, N = 4096, 512, 40
    wq = O.quantize(O.DT_Q8_0, weights(rng, M, K))
    x = rng.standard_normal((N, K)).astype(np.float32)
    y1 = run_mul_mat(b200, DType.Q8_0, wq, x, K, M)
    y4 = run_mul_mat(b200, DType.Q8_0, wq, x * np.float32(4), K, M)
    assert np.array_equal(y4, y1 * np.float32(4))


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
@pytest.mark.parametrize("K,M,N", [(2048, 1000, 64), (4096, 2048, 512)])
def test_repeated_calls_are_deterministic(b200, dt, K, M, N):
    """Same inputs, same bits: the GEMMs have no atomics and a fixed split-K
    reduction order, and their shared-memory stages must not race."""
    rng = np.random.default_rng(21)
    w = torch.from_numpy(O.quantize(QT[dt], weights(rng, M, K))).cuda()
    x = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda()
    outs = [ops.mul_mat(dt, w, x, K) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0])
def test_large_activations_stay_in_tolerance(b200, dt):
    """Activations far beyond the f16 range (rows up to 1e6, one row of
    zeros) through the large-N path: per-row power-of-two normalisation
    keeps every operand finite."""
    rng = np.random.default_rng(77)
    K, M, N = 1024, 160, 40
    wq = O.quantize(QT[dt], weights(rng, M, K))
    x = rng.standard_normal((N, K)).astype(np.float32)
    x *= np.logspace(-3, 6, N, dtype=np.float32)[:, None]
    x[7] = 0.0
    got = run_mul_mat(b200, dt, wq, x, K, M)
    want = O.mul_mat_quant_ref(QT[dt], wq, x, K)
    assert np.isfinite(got).all()
    # at these magnitudes any two f32 summation orders differ by a few ulps of
    # the partial sums, so the bound scales with sum_k |W||X| (the sum's
    # condition), not with |y|
    wd = np.abs(O.dequantize(QT[dt], wq, K)).astype(np.float64)
    xd = np.abs(O.dequantize(O.DT_Q8_0, O.quantize(O.DT_Q8_0, x), K)).astype(np.float64)
    bound = 1e-3 + 2e-5 * (xd @ wd.T)
    err = np.abs(got.astype(np.float64) - want)
    assert (err <= bound).all(), f"max err/bound {float((err / bound).max())}"


@pytest.mark.parametrize("d,ok", [(500.0, True), (600.0, False)])
def test_gemm_reports_weights_beyond_the_f16_range(b200, d, ok):
    """The Q8_0 GEMM splits every dequantized weight into two f16. A block
    scale whose products stay within the f16 range (500 * 127 = 63500) is
    exact; one that leaves it (600 * 127 = 76200) must fail loudly through
    the status word, not return infinities."""
    rng = np.random.default_rng(5)
    K, M, N = 512, 128, 16
    wq = O.quantize(O.DT_Q8_0, weights(rng, M, K)).copy()
    wq[5, 0:2] = np.frombuffer(np.float16(d).tobytes(), dtype=np.uint8)  # block 0 of row 5
    x = rng.standard_normal((N, K)).astype(np.float32)
    if ok:
        got = run_mul_mat(b200, DType.Q8_0, wq, x, K, M)
        good, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q8_0, wq, x, K))
        assert good, f"max abs err {err}"
    else:
        with pytest.raises(F.FemlError):
            run_mul_mat(b200, DType.Q8_0, wq, x, K, M)
        # the error was reported and cleared: the backend keeps working
        got = run_mul_mat(b200, DType.Q8_0, O.quantize(O.DT_Q8_0, weights(rng, M, K)), x, K, M)
        assert np.isfinite(got).all()


@pytest.mark.parametrize("off,v,ok", [(0, 60.0, True), (0, 80.0, False), (2, 1000.0, True), (2, 1100.0, False)])
def test_q4_k_gemm_reports_scales_beyond_the_f16_range(b200, off, v, ok):
    """The Q4_K GEMM (K % 512 == 0) splits d * (sc * q) into two f16, with
    sc * q <= 945, and carries -dmin * m (m <= 63) as f16 too: d up to
    65504 / 945 and dmin up to 65504 / 63 are exact, larger ones must fail
    loudly through the status word."""
    rng = np.random.default_rng(6)
    K, M, N = 1024, 128, 16
    wq = O.quantize(O.DT_Q4_K, weights(rng, M, K)).copy()
    wq[5, off:off + 2] = np.frombuffer(np.float16(v).tobytes(), dtype=np.uint8)  # super-block 0 of row 5
    x = rng.standard_normal((N, K)).astype(np.float32)
    if ok:
        got = run_mul_mat(b200, DType.Q4_K, wq, x, K, M)
        good, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q4_K, wq, x, K))
        assert good, f"max abs err {err}"
    else:
        with pytest.raises(F.FemlError):
            run_mul_mat(b200, DType.Q4_K, wq, x, K, M)
        got = run_mul_mat(b200, DType.Q4_K, O.quantize(O.DT_Q4_K, weights(rng, M, K)), x, K, M)
        assert np.isfinite(got).all()


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
@pytest.mark.parametrize("N", [100, 160])
def test_gemm_one_tile_properties(b200, dt, N):
    """A product of one column tile: at most 128 columns run the stacked
    two-MMA form, 129..192 the three-MMA form. Either way every column gets
    the same arithmetic (permuting the columns permutes the output bits) and
    scaling the activations by 8 scales the outputs by 8 exactly."""
    rng = np.random.default_rng(N)
    K, M = 1024, 384
    wq = O.quantize(QT[dt], weights(rng, M, K))
    x = rng.standard_normal((N, K)).astype(np.float32)
    wt = torch.from_numpy(wq).cuda()
    xt = torch.from_numpy(x).cuda()
    y = ops.mul_mat(dt, wt, xt, K)
    y8 = ops.mul_mat(dt, wt, xt * 8.0, K)
    perm = torch.from_numpy(rng.permutation(N)).cuda()
    yp = ops.mul_mat(dt, wt, xt[perm].contiguous(), K)
    torch.cuda.synchronize()
    assert torch.equal(y8, y * 8.0)
    assert torch.equal(yp, y[perm])
    ok, err = tol_ok(y.cpu().numpy(), O.mul_mat_quant_ref(QT[dt], wq, x, K))
    assert ok, f"max abs err {err}"


def test_gemm_tail_split_with_balanced_tiles(b200):
    """300 columns run as two balanced tiles of 160 + 140; 9600 weight rows
    give 75 x 2 = 150 tiles, 2 past one wave of 148, so the last weight-row
    tile row is split 4 ways in K and a reduction writes it (its column map
    follows the 160-column tiles). Every output against the oracle."""
    rng = np.random.default_rng(45)
    K, M, N = 2048, 9600, 300
    from feml_b200 import ops as _ops
    assert _ops.mul_mat_launches(DType.Q8_0, K, M, N) == 3  # quantizer, GEMM, tail reduction
    wq = O.quantize(O.DT_Q8_0, weights(rng, M, K))
    x = rng.standard_normal((N, K)).astype(np.float32)
    got = run_mul_mat(b200, DType.Q8_0, wq, x, K, M)
    ok, err = tol_ok(got, O.mul_mat_quant_ref(O.DT_Q8_0, wq, x, K))
    assert ok, f"max abs err {err}"
