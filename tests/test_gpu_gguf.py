"""GGUF weights through the reference-facing flow on the GPU: a file written
by llama.cpp's gguf-py is mapped by the library's reader, its tensors go to
HBM straight from the mapping (into a compiled plan's weight tensor, and as
one Weights buffer through buffer_from_host_ptr), and mul_mat on them
matches the oracle."""
import ctypes

import numpy as np
import pytest
import torch

import feml_b200 as F
from feml_b200 import DType, GraphBuilder, ops
from feml_b200.gguf import GGUFFile
from oracle import oracle as O
from tests.conftest import tol_ok

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as T  # noqa: E402

pytestmark = pytest.mark.gpu
K, M, N = 4096, 384, 3


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    rng = np.random.default_rng(77)
    p = tmp_path_factory.mktemp("gguf") / "m.gguf"
    w = gguf.GGUFWriter(str(p), "llama")
    w.add_custom_alignment(64)
    ws = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    q8 = gguf.quants.quantize(ws, T.Q8_0)
    q4k = O.quantize(O.DT_Q4_K, ws)
    w.add_tensor("blk.0.attn_q.weight", q8, raw_dtype=T.Q8_0)
    w.add_tensor("blk.0.ffn_down.weight", q4k, raw_dtype=T.Q4_K)
    w.add_tensor("output_norm.weight", ws[0])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    x = rng.standard_normal((N, K)).astype(np.float32)
    return p, {"blk.0.attn_q.weight": (DType.Q8_0, O.DT_Q8_0, q8), "blk.0.ffn_down.weight": (DType.Q4_K, O.DT_Q4_K, q4k)}, x


@pytest.mark.parametrize("name", ["blk.0.attn_q.weight", "blk.0.ffn_down.weight"])
def test_gguf_tensor_into_plan_then_mul_mat(b200, model, name):
    path, tensors, x = model
    dt, odt, wq = tensors[name]
    g = GraphBuilder()
    wi = g.weight(name, dt, [K, M])
    xi = g.input("x", DType.F32, [K, N])
    o = g.mul_mat(wi, xi)
    g.mark_output(o)
    plan = g.compile(b200)
    try:
        with GGUFFile(path) as f:
            f.write_to_plan(plan, b200, wi, name)
        plan.write_tensor(b200, xi, x)
        b200.graph_compute(plan)
        b200.synchronize()
        y = np.empty((N, M), np.float32)
        plan.read_tensor(b200, o, y)
        back = np.empty_like(wq)
        plan.read_tensor(b200, wi, back)
    finally:
        plan.release(b200)
    assert np.array_equal(back, wq)
    ok, err = tol_ok(y, O.mul_mat_quant_ref(odt, wq, x, K))
    assert ok, err


def test_gguf_upload_whole_data_section(b200, model):
    """buffer_from_host_ptr: one Weights buffer with the file's data section;
    the kernel-level mul_mat reads each tensor at its offset in HBM."""
    path, tensors, x = model
    with GGUFFile(path) as f:
        handle, offsets = f.upload(b200)
        total = max(t.offset + t.nbytes for t in f.tensors) - f.data_offset
    try:
        base, size = b200.device_ptr(handle)
        assert size == total
        xt = torch.from_numpy(x).cuda()
        for name, (dt, odt, wq) in tensors.items():
            back = np.empty(wq.nbytes, np.uint8)
            b200.read(handle, offsets[name], back)
            assert np.array_equal(back.reshape(wq.shape), wq)
            assert ops.mul_mat_workspace(dt, K, M, N) == 0
            y = torch.empty((N, M), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            b200.synchronize()
            rc = F._L.lib().feml_b200_mul_mat(int(dt), ctypes.c_void_p(base + offsets[name]), wq.shape[1],
                                              ctypes.c_void_p(xt.data_ptr()), K * 4, ctypes.c_void_p(y.data_ptr()),
                                              M * 4, K, M, N, None, 0, ctypes.c_void_p(b200.stream()))
            assert rc == 0, F._L.lib().feml_b200_last_error()
            b200.synchronize()
            ok, err = tol_ok(y.cpu().numpy(), O.mul_mat_quant_ref(odt, wq, x, K))
            assert ok, (name, err)
    finally:
        b200.release_buffer(handle)


def test_buffer_from_host_ptr_contract(b200):
    data = np.arange(4096, dtype=np.uint8)
    h = b200.buffer_from_host_ptr(data, data.nbytes, 1024)
    try:
        back = np.empty_like(data)
        b200.read(h, 0, back)
        assert np.array_equal(back, data)
    finally:
        b200.release_buffer(h)
    with pytest.raises(F.FemlError):
        b200.buffer_from_host_ptr(data, data.nbytes, data.nbytes + 1)  # tensor larger than the buffer
    dev = F.B200Device(0)
    with pytest.raises(F.FemlError):
        dev.buffer_from_host_ptr(data.ctypes.data, data.nbytes, 16)  # no owning backend named
    h = dev.buffer_from_host_ptr(data.ctypes.data, data.nbytes, 16, backend=b200)
    b200.release_buffer(h)
