"""ctypes wrapper over the C oracle -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference legs as the checker; never by the product package.
"""
import ctypes
import os

import numpy as np

from . import build_oracle

DT_F32, DT_Q4_0, DT_Q8_0, DT_Q4_K, DT_Q5_K, DT_Q6_K = 5, 7, 11, 15, 16, 17

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.OUT
        if not os.path.exists(path):
            path = build_oracle.build()
        L = ctypes.CDLL(path)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        for fn in ("oracle_quantize_row_q8_0", "oracle_dequantize_row_q8_0",
                   "oracle_quantize_row_q4_0", "oracle_dequantize_row_q4_0",
                   "oracle_quantize_row_q4_k", "oracle_dequantize_row_q4_k"):
            getattr(L, fn).restype = None
            getattr(L, fn).argtypes = [vp, vp, i64]
        L.oracle_row_bytes.restype = i64
        L.oracle_row_bytes.argtypes = [i32, i64]
        L.oracle_quantize_rows.restype = i32
        L.oracle_quantize_rows.argtypes = [i32, vp, vp, i64, i64]
        L.oracle_dequantize_rows.restype = i32
        L.oracle_dequantize_rows.argtypes = [i32, vp, vp, i64, i64]
        L.oracle_mul_mat_f32.restype = None
        L.oracle_mul_mat_f32.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, i32]
        L.oracle_block_dots.restype = i32
        L.oracle_block_dots.argtypes = [i32, vp, vp, vp, vp, i64, i64, i64]
        L.oracle_moe_route.restype = i64
        L.oracle_moe_route.argtypes = [vp, i64, i64, vp, vp, vp]
        L.oracle_q4k_scale_min.restype = None
        L.oracle_q4k_scale_min.argtypes = [i32, vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def row_bytes(dtype, k):
    return int(lib().oracle_row_bytes(dtype, k))


def quantize(dtype, x):
    """x: float32 [rows, k] (k contiguous) -> uint8 [rows, row_bytes]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    rows, k = x.shape
    out = np.zeros((rows, row_bytes(dtype, k)), dtype=np.uint8)
    assert lib().oracle_quantize_rows(dtype, _p(x), _p(out), rows, k) == 0
    return out


def dequantize(dtype, q, k):
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows = q.size // row_bytes(dtype, k)
    out = np.zeros((rows, k), dtype=np.float32)
    assert lib().oracle_dequantize_rows(dtype, _p(q), _p(out), rows, k) == 0
    return out


def mul_mat_f32(a, b, nthreads=None):
    """Reference mul_mat on f32: a [M, K] (row m = ggml column of ne=[K,M]),
    b [N, K] -> dst [N, M] (ggml dst ne=[M,N], M contiguous)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, K = a.shape
    N, K2 = b.shape
    assert K == K2
    c = np.zeros((N, M), dtype=np.float32)
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    lib().oracle_mul_mat_f32(_p(a), _p(b), _p(c), K, M, N, 4 * K, 4 * K, 4 * M, int(nthreads))
    return c


def quantize_q8_0_act(x):
    """Activations [N, K] f32 -> Q8_0 bytes [N, K/32*34] (quantize_row_q8_0)."""
    return quantize(DT_Q8_0, x)


def block_dots(dtype, w, xq, rows, K, N):
    """Per-block int32 sums -> (dots [rows, N, K/32], xsum [N, K/32])."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    nblk = K // 32
    out = np.zeros((rows, N, nblk), dtype=np.int32)
    xs = np.zeros((N, nblk), dtype=np.int32)
    assert lib().oracle_block_dots(dtype, _p(w), _p(xq), _p(out), _p(xs), rows, K, N) == 0
    return out, xs


def moe_route(ids, n_experts):
    """ids int32 [N, n_sel] (entry i = s + t*n_sel) -> (counts, offsets, rows, n_bad)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
    counts = np.zeros(n_experts, dtype=np.int32)
    offsets = np.zeros(n_experts, dtype=np.int32)
    rows = np.full(ids.size, -1, dtype=np.int32)
    bad = lib().oracle_moe_route(_p(ids), ids.size, n_experts, _p(counts), _p(offsets), _p(rows))
    return counts, offsets, rows[: ids.size - bad], int(bad)


def mul_mat_quant_ref(dtype, wq, x, K, quantize_act=True, nthreads=None):
    """O-Q8 (quantize_act) / O-F32 reference for a quantized weight:
    F32 mul_mat on dequant(W) and dequant(q8_0(x)) (or x itself).
    wq: uint8 [M, row_bytes]; x: f32 [N, K] -> [N, M]."""
    wf = dequantize(dtype, wq, K) if dtype != DT_F32 else np.ascontiguousarray(
        wq).view(np.float32).reshape(-1, K)
    xf = np.ascontiguousarray(x, dtype=np.float32)
    if quantize_act and dtype != DT_F32:
        xf = dequantize(DT_Q8_0, quantize(DT_Q8_0, xf), K)
    return mul_mat_f32(wf, xf, nthreads)


def mul_mat_id_ref(dtype, wq_experts, x, ids, K, quantize_act=True, nthreads=None):
    """ggml mul_mat_id: out[t, s, :] = W[ids[t, s]] . x[t]; wq_experts
    [E, M, row_bytes]; x [N, K]; ids [N, n_sel] -> [N, n_sel, M] f32.
    Slots with an out-of-range id are left at zero."""
    E, M = wq_experts.shape[0], wq_experts.shape[1]
    N, n_sel = ids.shape
    out = np.zeros((N, n_sel, M), dtype=np.float32)
    counts, offsets, rows, _ = moe_route(ids, E)
    for e in range(E):
        sl = rows[offsets[e]: offsets[e] + counts[e]]
        if sl.size == 0:
            continue
        toks = sl // n_sel
        y = mul_mat_quant_ref(dtype, wq_experts[e], x[toks], K, quantize_act, nthreads)
        out.reshape(N * n_sel, M)[sl] = y
    return out


def silu_f32(x):
    """SiLU as the plans define it (x / (1 + exp(-x))), in f32 -- the
    reference op (feml-core/src/op.rs:32) has no kernel to follow, so this is
    ggml's definition restated."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def add_f32(a, b):
    """The reference's broadcasting f32 add (feml-cpu/src/ops/elementwise.rs:30-96)."""
    return (np.asarray(a, dtype=np.float32) + np.asarray(b, dtype=np.float32)).astype(np.float32)
