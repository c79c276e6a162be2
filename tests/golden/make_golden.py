"""Regenerates the golden fixtures in tests/golden/ (run from the repo root:
`python tests/golden/make_golden.py`). Deterministic; the committed files are
its output.

Contents
 - mul_mat_ramp.json: the reference's F32 mul_mat known-answer tests,
   feml-cpu/tests/cpu_integration.rs:174-204 (w[i] = 0.1*i, x[i] = 0.01*i - 0.5,
   K=16, M=8, N=32) and feml-cuda/tests/cuda_integration.rs:246-278
   (w[i] = 0.3*i, x[i] = 0.05*i - 1.0). `want` is evaluated exactly as the
   reference test does: f32 products summed left to right from 0.0
   (`(0..16).map(|k| w[k + 16*m] * x[k + 16*n]).sum()`), here with numpy f32
   scalars, independent of the C oracle.
 - tables.json: the dtype size table, layout and planner known answers of
   feml-core/src/dtype.rs:124-182, layout.rs:68-113, planner.rs:284-398.
 - quant_vectors.npz: quantizer/dequantizer regression vectors produced by
   the oracle for seeded inputs and edge blocks (the reference has no quant
   arithmetic, so these pin the oracle against later changes, not against
   the reference).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402


def ramp_case(w_scale, x_scale, x_off, K=16, M=8, N=32):
    w = np.array([np.float32(i) * np.float32(w_scale) for i in range(K * M)], dtype=np.float32)
    x = np.array([np.float32(i) * np.float32(x_scale) - np.float32(x_off) for i in range(K * N)], dtype=np.float32)
    want = np.zeros(M * N, dtype=np.float32)
    for m in range(M):
        for n in range(N):
            acc = np.float32(0.0)
            for k in range(K):
                acc = np.float32(acc + np.float32(w[k + K * m] * x[k + K * n]))
            want[m + n * M] = acc
    return {"K": K, "M": M, "N": N, "w": w.tolist(), "x": x.tolist(), "want": want.tolist(),
            "w_bits": w.view(np.uint32).tolist(), "x_bits": x.view(np.uint32).tolist(),
            "want_bits": want.view(np.uint32).tolist(), "tolerance": 1e-3}


def main():
    ramps = {
        "cpu_integration_mul_mat_matches_reference": ramp_case(0.1, 0.01, 0.5),
        "cuda_integration_cpu_and_cuda_agree": ramp_case(0.3, 0.05, 1.0),
    }
    with open(os.path.join(HERE, "mul_mat_ramp.json"), "w") as f:
        json.dump(ramps, f)

    tables = {
        # dtype.rs:124-182 (name, block_size, type_size, quantized)
        "dtype": [["I8", 1, 1, False], ["I16", 1, 2, False], ["I32", 1, 4, False], ["I64", 1, 8, False],
                  ["F16", 1, 2, False], ["F32", 1, 4, False], ["F64", 1, 8, False],
                  ["Q4_0", 32, 18, True], ["Q4_1", 32, 20, True], ["Q5_0", 32, 22, True],
                  ["Q5_1", 32, 24, True], ["Q8_0", 32, 34, True], ["Q8_1", 32, 36, True],
                  ["Q2_K", 256, 84, True], ["Q3_K", 256, 110, True], ["Q4_K", 256, 144, True],
                  ["Q5_K", 256, 176, True], ["Q6_K", 256, 210, True], ["Q8_K", 256, 292, True]],
        "row_size": [["F32", 4096, 16384], ["F16", 3, 6], ["Q4_0", 64, 36], ["Q4_K", 256, 144]],
        "row_size_misaligned": [["Q4_0", 33]],
        # layout.rs:68-113 (dtype, shape, stride prefix, nbytes)
        "layout": [["F32", [2, 3], [4, 8, 24], 24], ["F32", [100], [4], 400],
                   ["F32", [1, 3, 224, 224], [4], 3 * 224 * 224 * 4], ["Q4_0", [64], [18], 36],
                   ["Q4_K", [256], [144], 144], ["Q4_0", [64, 2], [18, 36], 72]],
        # planner.rs tests: compute_size expectations
        "planner": {"diamond_shared_source": 64, "inplace_op_reuses_sole_parent": 32,
                    "compute_tensor_reuses_freed_slot": 128},
    }
    with open(os.path.join(HERE, "tables.json"), "w") as f:
        json.dump(tables, f, indent=1)

    rng = np.random.default_rng(1234)
    K = 512
    x = (rng.standard_normal((6, K)) * 0.7).astype(np.float32)
    # edge blocks: all zero, a negative zero, exact .5 ties of x*(1/d), one
    # huge value, constant block, alternating sign maxima
    x[0, :32] = 0.0
    x[0, 32:64] = -0.0
    x[1, :32] = np.arange(32, dtype=np.float32) - 15.5
    x[1, 32:64] = 0.0
    x[1, 40] = 1000.0
    x[2, :32] = 3.0
    x[2, 32:64] = np.where(np.arange(32) % 2 == 0, 2.0, -2.0).astype(np.float32)
    x[3, :256] = np.abs(x[3, :256])  # Q4_K super-block with no negative values
    out = {"x": x}
    for name, dt in (("q8_0", O.DT_Q8_0), ("q4_0", O.DT_Q4_0), ("q4_k", O.DT_Q4_K)):
        q = O.quantize(dt, x)
        out[name] = q
        out[name + "_deq"] = O.dequantize(dt, q, K)
    np.savez_compressed(os.path.join(HERE, "quant_vectors.npz"), **out)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
