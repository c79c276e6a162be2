"""CPU: pins the oracle (oracle/feml_oracle.c) before anything is checked
against it.

 - F32 mul_mat: bit-exact against the reference's own known-answer tests
   (feml-cpu/tests/cpu_integration.rs:174-204,
   feml-cuda/tests/cuda_integration.rs:246-278), whose expected values are
   sequential f32 sums.
 - Quant formats: the oracle's dequantizers against an independent numpy
   restatement of the published ggml block layouts, and its quantizers
   against the committed regression vectors. The reference has no quant
   arithmetic, so this pins the oracle's reading of the formats, not the
   reference (parity for quantized types is unpinned by the reference).
   The Q8_0 / Q4_0 quantizers and Q8_0 / Q4_0 / Q4_K dequantizers are also
   pinned byte for byte to llama.cpp's own Python implementation of the
   formats (gguf-py): against its committed vectors
   (tests/golden/ggufpy_vectors.npz) and, where the package is installed,
   live on fresh inputs.
 - Routing: against a numpy stable sort.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _ramp(name):
    with open(os.path.join(GOLD, "mul_mat_ramp.json")) as f:
        c = json.load(f)[name]
    K, M, N = c["K"], c["M"], c["N"]
    w = np.array(c["w_bits"], dtype=np.uint32).view(np.float32).reshape(M, K)
    x = np.array(c["x_bits"], dtype=np.uint32).view(np.float32).reshape(N, K)
    want = np.array(c["want_bits"], dtype=np.uint32).view(np.float32).reshape(N, M)
    return w, x, want


@pytest.mark.parametrize("name", ["cpu_integration_mul_mat_matches_reference", "cuda_integration_cpu_and_cuda_agree"])
@pytest.mark.parametrize("threads", [1, 3])
def test_oracle_mul_mat_matches_reference_known_answers(name, threads):
    w, x, want = _ramp(name)
    got = O.mul_mat_f32(w, x, nthreads=threads)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_oracle_mul_mat_sequential_accumulation():
    # the oracle must accumulate in k order in f32 (no reassociation, no FMA)
    rng = np.random.default_rng(7)
    w = rng.standard_normal((5, 301)).astype(np.float32)
    x = rng.standard_normal((3, 301)).astype(np.float32)
    got = O.mul_mat_f32(w, x)
    for n in range(3):
        for m in range(5):
            acc = np.float32(0)
            for k in range(301):
                acc = np.float32(acc + np.float32(w[m, k] * x[n, k]))
            assert got[n, m] == acc


# ---- independent numpy restatement of the ggml block formats --------------
def np_f16(b0, b1):
    return np.frombuffer(bytes([b0, b1]), dtype=np.float16)[0].astype(np.float32)


def np_deq_q8_0(row, k):
    out = np.zeros(k, np.float32)
    for i in range(k // 32):
        blk = row[34 * i: 34 * i + 34]
        d = np_f16(blk[0], blk[1])
        out[32 * i: 32 * i + 32] = blk[2:].view(np.int8).astype(np.float32) * d
    return out


def np_deq_q4_0(row, k):
    out = np.zeros(k, np.float32)
    for i in range(k // 32):
        blk = row[18 * i: 18 * i + 18]
        d = np_f16(blk[0], blk[1])
        qs = blk[2:]
        out[32 * i: 32 * i + 16] = ((qs & 0x0F).astype(np.int32) - 8).astype(np.float32) * d
        out[32 * i + 16: 32 * i + 32] = ((qs >> 4).astype(np.int32) - 8).astype(np.float32) * d
    return out


def np_q4k_scale_min(j, s):
    if j < 4:
        return int(s[j] & 63), int(s[j + 4] & 63)
    return int((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4)), int((s[j + 4] >> 4) | ((s[j] >> 6) << 4))


def np_deq_q4_k(row, k):
    out = np.zeros(k, np.float32)
    for i in range(k // 256):
        blk = row[144 * i: 144 * i + 144]
        d, dmin = np_f16(blk[0], blk[1]), np_f16(blk[2], blk[3])
        sc, qs = blk[4:16], blk[16:]
        for j in range(8):
            s, m = np_q4k_scale_min(j, sc)
            nib = qs[32 * (j // 2): 32 * (j // 2) + 32]
            q = (nib & 0xF) if j % 2 == 0 else (nib >> 4)
            d1, m1 = np.float32(d * np.float32(s)), np.float32(dmin * np.float32(m))
            out[256 * i + 32 * j: 256 * i + 32 * j + 32] = (d1 * q.astype(np.float32)) - m1
    return out


def np_quant_q8_0(x):
    k = x.size
    out = bytearray()
    for i in range(k // 32):
        b = x[32 * i: 32 * i + 32].astype(np.float32)
        amax = np.float32(np.max(np.abs(b)))
        d = np.float32(amax / np.float32(127))
        idv = np.float32(np.float32(1) / d) if d != 0 else np.float32(0)
        v = (b * idv).astype(np.float32).astype(np.float64)
        q = (np.sign(v) * np.floor(np.abs(v) + 0.5)).astype(np.int8)  # half away from zero
        out += np.float16(d).tobytes() + q.tobytes()
    return np.frombuffer(bytes(out), np.uint8)


DEQ = {O.DT_Q8_0: np_deq_q8_0, O.DT_Q4_0: np_deq_q4_0, O.DT_Q4_K: np_deq_q4_k}


@pytest.mark.parametrize("dt", [O.DT_Q8_0, O.DT_Q4_0, O.DT_Q4_K])
def test_oracle_dequant_matches_format_restatement(dt):
    gv = np.load(os.path.join(GOLD, "quant_vectors.npz"))
    x = gv["x"]
    q = O.quantize(dt, x)
    deq = O.dequantize(dt, q, x.shape[1])
    for r in range(x.shape[0]):
        ref = DEQ[dt](q[r], x.shape[1])
        assert np.array_equal(deq[r].view(np.uint32), ref.view(np.uint32)), r


def test_oracle_quantize_q8_0_matches_restatement():
    gv = np.load(os.path.join(GOLD, "quant_vectors.npz"))
    x = gv["x"]
    q = O.quantize(O.DT_Q8_0, x)
    for r in range(x.shape[0]):
        assert np.array_equal(q[r], np_quant_q8_0(x[r])), r


@pytest.mark.parametrize("name,dt", [("q8_0", O.DT_Q8_0), ("q4_0", O.DT_Q4_0), ("q4_k", O.DT_Q4_K)])
def test_oracle_quantizers_match_committed_vectors(name, dt):
    gv = np.load(os.path.join(GOLD, "quant_vectors.npz"))
    q = O.quantize(dt, gv["x"])
    assert np.array_equal(q, gv[name])
    deq = O.dequantize(dt, q, gv["x"].shape[1])
    assert np.array_equal(deq.view(np.uint32), gv[name + "_deq"].view(np.uint32))


def _same_blocks(got, want, x, block_bytes):
    """Quantized rows equal block by block, except that for a block whose
    inputs are all zeros the scale may be +0 or -0: the Q4_0 quantizer takes
    `max` as the first value of largest magnitude starting from +0 (ggml's C
    reference does the same), gguf-py's numpy version takes the block's first
    element, so an all-(-0) block gives d = -0 here and +0 there."""
    g = got.reshape(got.shape[0], -1, block_bytes)
    w = want.reshape(want.shape[0], -1, block_bytes)
    zero = np.all(x.reshape(x.shape[0], -1, 32) == 0, axis=-1)
    assert np.array_equal(g[..., 2:], w[..., 2:])
    same_d = np.all(g[..., :2] == w[..., :2], axis=-1)
    dg = g[..., 0].astype(np.uint16) | (g[..., 1].astype(np.uint16) << 8)
    dw = w[..., 0].astype(np.uint16) | (w[..., 1].astype(np.uint16) << 8)
    signed_zero = zero & ((dg & 0x7FFF) == 0) & ((dw & 0x7FFF) == 0)
    assert np.all(same_d | signed_zero)


@pytest.mark.parametrize("name,dt", [("q8_0", O.DT_Q8_0), ("q4_0", O.DT_Q4_0), ("q4_k", O.DT_Q4_K),
                                     ("q5_k", O.DT_Q5_K), ("q6_k", O.DT_Q6_K)])
def test_oracle_matches_ggufpy_vectors(name, dt):
    gv = np.load(os.path.join(GOLD, "ggufpy_vectors.npz"))
    if not name.endswith("_k"):  # gguf-py has no K-quant quantizers; its dequantizers pin the layouts
        _same_blocks(O.quantize(dt, gv["x"]), gv[name], gv["x"], 34 if name == "q8_0" else 18)
    deq = O.dequantize(dt, gv[name], gv[name + "_deq"].shape[1])
    assert np.array_equal(deq.view(np.uint32), gv[name + "_deq"].view(np.uint32))


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_matches_ggufpy_live(seed):
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((16, 1024)) * rng.uniform(0.01, 10.0, (16, 1))).astype(np.float32)
    for dt, t in ((O.DT_Q8_0, T.Q8_0), (O.DT_Q4_0, T.Q4_0)):
        q = gguf.quants.quantize(x, t)
        _same_blocks(O.quantize(dt, x), q, x, 34 if dt == O.DT_Q8_0 else 18)
        assert np.array_equal(O.dequantize(dt, q, 1024).view(np.uint32),
                              gguf.quants.dequantize(q, t).astype(np.float32).view(np.uint32))
    for dt, t in ((O.DT_Q4_K, T.Q4_K), (O.DT_Q5_K, T.Q5_K), (O.DT_Q6_K, T.Q6_K)):
        q = O.quantize(dt, x)
        assert np.array_equal(O.dequantize(dt, q, 1024).view(np.uint32),
                              gguf.quants.dequantize(q, t).astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("dt,levels", [(O.DT_Q4_K, 15), (O.DT_Q5_K, 31), (O.DT_Q6_K, 31)])
def test_k_quantizers_round_trip(dt, levels):
    """The project's K-quant quantizers (parity-unpinned schemes) stay within
    about one quantization step of the input, zero blocks stay zero."""
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((8, 2048)) * 0.02).astype(np.float32)
    x[0, :256] = 0.0
    y = O.dequantize(dt, O.quantize(dt, x), 2048)
    assert np.all(y[0, :256] == 0.0)
    step = 2 * np.abs(x).max() / levels
    assert np.abs(y - x).max() <= 1.5 * step


def test_q8_0_edge_blocks():
    x = np.zeros(96, np.float32)
    x[32:64] = -0.0
    x[64:96] = np.arange(32, dtype=np.float32) - 15.5
    q = O.quantize(O.DT_Q8_0, x)[0]
    assert q[0] == 0 and q[1] == 0 and not q[2:34].any()       # all-zero block: d = 0, q = 0
    assert not q[36:68].any()                                    # -0.0 block quantizes to zeros
    d = np.frombuffer(q[68:70].tobytes(), np.float16)[0]
    assert d == np.float16(np.float32(15.5) / np.float32(127))
    qs = q[70:102].view(np.int8)
    assert qs[0] == -127 and qs[31] == 127                       # amax maps to +-127


def test_q4_0_first_max_rule():
    # the signed value of largest magnitude, first occurrence, sets d = max / -8
    x = np.zeros(32, np.float32)
    x[3], x[9] = -4.0, 4.0
    q = O.quantize(O.DT_Q4_0, x)[0]
    d = np.frombuffer(q[0:2].tobytes(), np.float16)[0]
    assert d == np.float16(0.5)   # -4 / -8
    x[3], x[9] = 4.0, -4.0
    q = O.quantize(O.DT_Q4_0, x)[0]
    assert np.frombuffer(q[0:2].tobytes(), np.float16)[0] == np.float16(-0.5)


def test_block_dots_definition():
    rng = np.random.default_rng(3)
    K, M, N = 512, 3, 2
    w = rng.standard_normal((M, K)).astype(np.float32)
    x = rng.standard_normal((N, K)).astype(np.float32)
    xq = O.quantize(O.DT_Q8_0, x)
    xi = np.stack([xq[n].reshape(-1, 34)[:, 2:].view(np.int8).reshape(-1).astype(np.int64) for n in range(N)])
    for dt in (O.DT_Q8_0, O.DT_Q4_0, O.DT_Q4_K):
        wq = O.quantize(dt, w)
        dots, xs = O.block_dots(dt, wq, xq, M, K, N)
        for m in range(M):
            if dt == O.DT_Q8_0:
                wi = wq[m].reshape(-1, 34)[:, 2:].view(np.int8).reshape(-1).astype(np.int64)
            elif dt == O.DT_Q4_0:
                b = wq[m].reshape(-1, 18)[:, 2:]
                wi = np.concatenate([(b & 15).astype(np.int64) - 8, (b >> 4).astype(np.int64) - 8], axis=1).reshape(-1)
            else:
                sbs = wq[m].reshape(-1, 144)[:, 16:]
                parts = []
                for sb in sbs:
                    for j in range(8):
                        nib = sb[32 * (j // 2): 32 * (j // 2) + 32]
                        parts.append(((nib & 15) if j % 2 == 0 else (nib >> 4)).astype(np.int64))
                wi = np.concatenate(parts)
            for n in range(N):
                want = (wi * xi[n]).reshape(-1, 32).sum(axis=1)
                assert np.array_equal(dots[m, n], want)
        assert np.array_equal(xs, xi.reshape(N, -1, 32).sum(axis=2))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_moe_route_is_stable_sort(seed):
    rng = np.random.default_rng(seed)
    N, n_sel, E = 257, 2, 8
    ids = np.stack([rng.permutation(E)[:n_sel] for _ in range(N)]).astype(np.int32)
    counts, offsets, rows, bad = O.moe_route(ids, E)
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")
    assert bad == 0
    assert np.array_equal(rows, order.astype(np.int32))
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(counts)[:-1]]))


def test_moe_route_skips_bad_ids():
    ids = np.array([[0, 9], [-1, 1], [1, 0]], dtype=np.int32)
    counts, offsets, rows, bad = O.moe_route(ids, 2)
    assert bad == 2
    assert list(counts) == [2, 2] and list(rows) == [0, 5, 3, 4]


def test_mul_mat_id_ref_shapes():
    rng = np.random.default_rng(5)
    E, M, K, N, n_sel = 3, 16, 64, 5, 2
    w = rng.standard_normal((E, M, K)).astype(np.float32)
    wq = np.stack([O.quantize(O.DT_Q8_0, w[e]) for e in range(E)])
    x = rng.standard_normal((N, K)).astype(np.float32)
    ids = np.array([[0, 2], [1, 0], [2, 1], [0, 1], [2, 0]], dtype=np.int32)
    out = O.mul_mat_id_ref(O.DT_Q8_0, wq, x, ids, K)
    for t in range(N):
        for s in range(n_sel):
            want = O.mul_mat_quant_ref(O.DT_Q8_0, wq[ids[t, s]], x[t:t + 1], K)[0]
            assert np.array_equal(out[t, s], want)
