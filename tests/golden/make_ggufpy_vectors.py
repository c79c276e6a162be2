"""Regenerates tests/golden/ggufpy_vectors.npz (run from the repo root:
`python tests/golden/make_ggufpy_vectors.py`). Deterministic.

The vectors come from llama.cpp's Python package `gguf` (gguf-py, the
ecosystem's published numpy implementation of the ggml block formats,
installed in this image), not from this repository's oracle, so the oracle's
Q8_0 / Q4_0 quantizers and Q8_0 / Q4_0 / Q4_K dequantizers are pinned to an
independent implementation of the formats:
 - x: f32 inputs with edge blocks (zero, negative zero, exact .5 ties of
   x*(1/d), one huge value, constant block, alternating-sign maxima);
 - q8_0, q4_0: gguf.quants.quantize(x, ...) bytes, and *_deq their
   gguf.quants.dequantize values;
 - q4_k, q5_k, q6_k: seeded blocks with finite f16 scales and random
   packed scales, mins, high bits and nibbles; *_deq: gguf.quants.dequantize.
"""
import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    import importlib.metadata as md
    rng = np.random.default_rng(2024)
    K = 512
    x = (rng.standard_normal((8, K)) * 0.5).astype(np.float32)
    x[0, :32] = 0.0
    x[0, 32:64] = -0.0
    x[1, :32] = np.arange(32, dtype=np.float32) - 15.5
    x[1, 32:64] = 0.0
    x[1, 40] = 1000.0
    x[2, :32] = 3.0
    x[2, 32:64] = np.where(np.arange(32) % 2 == 0, 2.0, -2.0).astype(np.float32)
    x[3, 64:96] = -7.0
    out = {"x": x, "gguf_version": np.array(md.version("gguf"))}
    for name, t in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        q = quants.quantize(x, t)
        out[name] = q
        out[name + "_deq"] = quants.dequantize(q, t).astype(np.float32)
    rows, nsb = 8, 2
    for name, t, nbytes, d_at, nd in (("q4_k", T.Q4_K, 144, 0, 2), ("q5_k", T.Q5_K, 176, 0, 2),
                                      ("q6_k", T.Q6_K, 210, 208, 1)):
        blk = rng.integers(0, 256, (rows, nsb, nbytes), dtype=np.uint8)
        d = (rng.uniform(0.5, 2.0, (rows, nsb, nd)) * 1e-3).astype(np.float16)
        blk[:, :, d_at:d_at + 2 * nd] = d.view(np.uint8).reshape(rows, nsb, 2 * nd)
        q = blk.reshape(rows, nsb * nbytes)
        out[name] = q
        out[name + "_deq"] = quants.dequantize(q, t).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "ggufpy_vectors.npz"), **out)
    print("wrote ggufpy_vectors.npz")


if __name__ == "__main__":
    main()
