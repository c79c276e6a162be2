"""Shared helpers of the GPU parity tests: run mul_mat / mul_mat_id through the
reference-facing flow (GraphBuilder -> compile -> graph_compute on the B200
backend, all through the C ABI) and compare with the oracle."""
import numpy as np

import feml_b200 as F
from feml_b200 import DType, GraphBuilder


def run_mul_mat(be, wtype, wbytes, x, K, M):
    """wbytes: uint8 [M, row_bytes] (F32: float32 [M, K]); x: f32 [N, K] -> f32 [N, M]."""
    N = x.shape[0]
    g = GraphBuilder()
    w = g.weight("w", wtype, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    o = g.mul_mat(w, xi)
    g.mark_output(o)
    plan = g.compile(be)
    try:
        plan.write_tensor(be, w, np.ascontiguousarray(wbytes))
        plan.write_tensor(be, xi, np.ascontiguousarray(x, dtype=np.float32))
        be.graph_compute(plan)
        be.synchronize()
        out = np.empty((N, M), dtype=np.float32)
        plan.read_tensor(be, o, out)
    finally:
        plan.release(be)
    return out


def run_mul_mat_id(be, wtype, wbytes, x, ids, K, M, check_sync=True):
    """wbytes: [E, M, row_bytes]; x: f32 [N, K]; ids int32 [N, n_sel] -> [N, n_sel, M]."""
    E = wbytes.shape[0]
    N, n_sel = ids.shape
    g = GraphBuilder()
    w = g.weight("w", wtype, [K, M, E])
    xi = g.input("x", DType.F32, [K, N])
    ii = g.input("ids", DType.I32, [n_sel, N])
    o = g.mul_mat_id(w, xi, ii, n_sel)
    g.mark_output(o)
    plan = g.compile(be)
    err = None
    try:
        plan.write_tensor(be, w, np.ascontiguousarray(wbytes))
        plan.write_tensor(be, xi, np.ascontiguousarray(x, dtype=np.float32))
        plan.write_tensor(be, ii, np.ascontiguousarray(ids, dtype=np.int32))
        be.graph_compute(plan)
        try:
            be.synchronize()
        except F.FemlError as e:
            if check_sync:
                raise
            err = e
        out = np.empty((N, n_sel, M), dtype=np.float32)
        plan.read_tensor(be, o, out)
    finally:
        plan.release(be)
    return (out, err) if not check_sync else out


def weights(rng, M, K, std=0.02):
    return (rng.standard_normal((M, K)) * std).astype(np.float32)
