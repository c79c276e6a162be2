"""CPU: the host side of the boundary (C++ mirror of feml-core inside
libfeml_b200.so) against the reference's own unit tests, plus the C-ABI
export list. No GPU is touched: compile() is driven through Python test
doubles, as the reference drives it through DummyBackend / Stub
(feml-core/src/graph.rs:453-541)."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

import feml_b200 as F
from feml_b200 import BufferUsage, DType, FemlError, GraphBuilder, Op, TensorFlags

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


class DummyBackend(F.Backend):
    """graph.rs:453-503: records buffer sizes, executes nothing."""

    def __init__(self):
        self.buffers = {}
        self.next = 1
        self.data = {}

    def name(self):
        return "dummy"

    def create_buffer(self, size, usage):
        h = self.next
        self.next += 1
        self.buffers[h] = size
        self.data[h] = bytearray(size)
        return h

    def release_buffer(self, h):
        if h not in self.buffers:
            raise FemlError("msg", "release_buffer: unknown")
        del self.buffers[h]

    def write(self, h, off, data):
        if h not in self.data or off + len(data) > len(self.data[h]):
            raise FemlError("msg", "write: overflow")
        self.data[h][off:off + len(data)] = data

    def read(self, h, off, n):
        if h not in self.data or off + n > len(self.data[h]):
            raise FemlError("msg", "read: overflow")
        return bytes(self.data[h][off:off + n])

    def fill(self, h, off, v, n):
        self.data[h][off:off + n] = bytes([v]) * n

    def graph_compute(self, plan):
        pass

    def supports_op(self, op, dts):
        return True


class StubBackend(F.Backend):
    """graph.rs:506-541: any allocation is a test failure."""

    def name(self):
        return "stub"

    def create_buffer(self, size, usage):
        raise AssertionError("compile must reject before allocating")

    def supports_op(self, op, dts):
        return False


def tables():
    with open(os.path.join(GOLD, "tables.json")) as f:
        return json.load(f)


# ---- dtype / layout (dtype.rs:124-182, layout.rs:68-113) ------------------
def test_dtype_table_matches_ggml():
    for name, bs, ts, q in tables()["dtype"]:
        d = DType[name]
        assert (d.block_size, d.type_size, d.is_quantized) == (bs, ts, q), name


def test_row_size():
    for name, n, want in tables()["row_size"]:
        assert DType[name].row_size(n) == want
    for name, n in tables()["row_size_misaligned"]:
        with pytest.raises(FemlError):
            DType[name].row_size(n)


def test_layout_strides_and_nbytes():
    for name, shape, stride, nbytes in tables()["layout"]:
        nb = F.layout_new(DType[name], shape)
        assert nb[: len(stride)] == stride, (name, shape)
        assert F.layout_nbytes(DType[name], shape, nb) == nbytes, (name, shape)


def test_shape_validation():
    g = GraphBuilder()
    with pytest.raises(FemlError) as e:
        g.input("a", DType.F32, [0, 2])
    assert e.value.kind == "shape"
    with pytest.raises(FemlError):
        g.input("a", DType.F32, [1, 2, 3, 4, 5])


# ---- planner (planner.rs:284-398) -----------------------------------------
IN, OUT, W = TensorFlags.INPUT, TensorFlags.OUTPUT, TensorFlags.WEIGHT


def T(id, shape, flags=0, op=Op.NONE, srcs=(), view_src=0, view_offset=0, dtype=DType.F32):
    return {"id": id, "shape": shape, "flags": flags, "op": op, "srcs": list(srcs), "view_src": view_src,
            "view_offset": view_offset, "dtype": dtype}


def test_planner_diamond_shared_source():
    ts = [T(1, [4], IN), T(2, [4], IN), T(3, [4], 0, Op.MUL, [1, 2]), T(4, [4], 0, Op.MUL, [1, 3])]
    a, _, cs = F.planner_plan(ts, [2, 3])
    assert a[1][1] != a[2][1]
    assert a[2][1] == a[3][1], "c reuses single-child b"
    assert a[1][1] == a[4][1], "d reuses a (live child count)"
    assert cs == tables()["planner"]["diamond_shared_source"]


def test_planner_inplace_reuses_sole_parent():
    ts = [T(1, [8], IN), T(2, [8], 0, Op.SILU, [1])]
    a, _, cs = F.planner_plan(ts, [1])
    assert a[1][1] == a[2][1]
    assert cs == tables()["planner"]["inplace_op_reuses_sole_parent"]


def test_planner_inplace_reused_parent_not_freed():
    ts = [T(1, [8], IN), T(2, [8], 0, Op.SILU, [1]), T(3, [8], OUT, Op.COPY, [2])]
    a, _, _ = F.planner_plan(ts, [1, 2])
    assert a[1][1] == a[2][1]
    assert a[3][1] != a[1][1], "output must get its own slot"


def test_planner_non_inplace_op_gets_own_slot():
    ts = [T(1, [4, 4], W), T(2, [4, 1], IN), T(3, [4, 1], 0, Op.MUL_MAT, [1, 2])]
    a, _, _ = F.planner_plan(ts, [2])
    assert a[1][0] == 0 and a[2][0] == 1
    assert a[3][1] != a[2][1]


def test_planner_view_shares_source_buffer():
    ts = [T(1, [8], IN), T(2, [4], 0, Op.NONE, [], view_src=1, view_offset=16), T(3, [4], 0, Op.COPY, [2])]
    a, _, _ = F.planner_plan(ts, [2])
    assert a[2][0] == a[1][0]
    assert a[2][1] == a[1][1] + 16


def test_planner_compute_tensor_reuses_freed_slot():
    ts = [T(1, [16], IN), T(2, [16], IN), T(3, [16], 0, Op.MUL, [1, 2]), T(4, [16], 0, Op.MUL, [3, 2])]
    a, _, cs = F.planner_plan(ts, [2, 3])
    assert cs == tables()["planner"]["compute_tensor_reuses_freed_slot"]
    assert a[4][1] in (a[1][1], a[2][1])


def test_planner_offsets_are_32_aligned_for_quant_layouts():
    ts = [T(1, [4096, 4096], W, dtype=DType.Q8_0), T(2, [4096, 1], IN), T(3, [4096, 1], OUT, Op.MUL_MAT, [1, 2])]
    a, ws, cs = F.planner_plan(ts, [2])
    assert ws == 4096 * 4352
    assert all(off % 32 == 0 for _, off in a.values())


# ---- GraphBuilder / compile (graph.rs:505-697) -----------------------------
def test_compile_rejects_unsupported_op_before_allocating():
    g = GraphBuilder()
    x = g.input("x", DType.F32, [4])
    s = g.silu(x)
    g.mark_output(s)
    with pytest.raises(FemlError) as e:
        g.compile(StubBackend())
    assert "does not support op silu" in str(e.value)


def test_build_chain_and_compile():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    c = g.mul(a, b)
    g.mark_output(c)
    assert g.tensor(c).op == Op.MUL
    assert g.outputs() == [c]
    plan = g.compile(DummyBackend())
    assert len(plan.nodes) == 1 and len(plan.tensors) == 3
    assert plan.find(c) is not None


def test_mul_mat_shape_check():
    g = GraphBuilder()
    w = g.weight("w", DType.F32, [16, 8])
    x = g.input("x", DType.F32, [16, 32])
    out = g.mul_mat(w, x)
    assert g.tensor(out).shape[:2] == [8, 32]
    assert g.tensor(out).dtype == DType.F32


def test_mul_mat_rejects_inner_mismatch():
    g = GraphBuilder()
    w = g.weight("w", DType.F32, [16, 8])
    x = g.input("x", DType.F32, [32, 32])
    with pytest.raises(FemlError) as e:
        g.mul_mat(w, x)
    assert e.value.kind == "shape"


@pytest.mark.parametrize("dt", [DType.Q8_0, DType.Q4_0, DType.Q4_K])
def test_mul_mat_accepts_quant_weights_f32_output(dt):
    g = GraphBuilder()
    K = 512
    w = g.weight("w", dt, [K, 64])
    x = g.input("x", DType.F32, [K, 3])
    out = g.mul_mat(w, x)
    t = g.tensor(out)
    assert t.dtype == DType.F32 and t.shape[:2] == [64, 3]
    assert g.tensor(w).stride[1] == dt.row_size(K)


def test_mul_mat_rejects_unsupported_dtypes():
    g = GraphBuilder()
    w = g.weight("w", DType.Q5_0, [64, 4])
    x = g.input("x", DType.F32, [64, 2])
    with pytest.raises(FemlError) as e:
        g.mul_mat(w, x)
    assert e.value.kind == "unsupported"
    w2 = g.weight("w2", DType.Q8_0, [64, 4])
    x2 = g.input("x2", DType.F16, [64, 2])
    with pytest.raises(FemlError):
        g.mul_mat(w2, x2)
    w3 = g.weight("w3", DType.Q4_K, [288, 4])  # K not a multiple of 256
    x3 = g.input("x3", DType.F32, [288, 2])
    with pytest.raises(FemlError) as e:
        g.mul_mat(w3, x3)
    assert e.value.kind == "shape"


def test_mul_rejects_dtype_mismatch():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.I32, [4])
    with pytest.raises(FemlError):
        g.mul(a, b)


def test_compile_requires_output():
    with pytest.raises(FemlError):
        GraphBuilder().compile(DummyBackend())


def test_view_bounds_checked():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [8])
    with pytest.raises(FemlError):
        g.view(a, 24, [4])
    with pytest.raises(FemlError):
        g.view(a, 2, [4])  # not 4-byte aligned
    v = g.view(a, 16, [4])
    assert g.tensor(v).op == Op.VIEW


def test_topo_order_respects_dependencies():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    c = g.mul(a, b)
    d = g.mul(a, c)
    g.mark_output(d)
    plan = g.compile(DummyBackend())
    order = [plan.tensors[i].id for i in plan.nodes]
    assert order.index(c) < order.index(d)


def test_diamond_executes_source_once():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    c = g.mul(a, b)
    d = g.add(c, c)
    g.mark_output(d)
    assert len(g.compile(DummyBackend()).nodes) == 2


def test_mul_mat_id_ggml_semantics():
    g = GraphBuilder()
    w = g.weight("w", DType.Q8_0, [256, 64, 8])
    x = g.input("x", DType.F32, [256, 32])
    ids = g.input("ids", DType.I32, [2, 32])
    out = g.mul_mat_id(w, x, ids, 2)
    t = g.tensor(out)
    assert t.shape[:3] == [64, 2, 32] and t.dtype == DType.F32
    bad = g.input("bad", DType.I32, [3, 32])
    with pytest.raises(FemlError):
        g.mul_mat_id(w, x, bad, 2)
    badf = g.input("badf", DType.F32, [2, 32])
    with pytest.raises(FemlError):
        g.mul_mat_id(w, x, badf, 2)
    with pytest.raises(FemlError):
        g.mul_mat_id(w, x, ids, 9)


def test_compile_places_weights_and_activations():
    g = GraphBuilder()
    w = g.weight("w", DType.Q4_0, [4096, 11008])
    x = g.input("x", DType.F32, [4096, 512])
    out = g.mul_mat(w, x)
    g.mark_output(out)
    be = DummyBackend()
    plan = g.compile(be)
    assert [b.usage for b in plan.buffers] == [BufferUsage.WEIGHTS, BufferUsage.COMPUTE]
    assert plan.buffers[0].size == 11008 * 2304
    pw, px, po = plan.find(w), plan.find(x), plan.find(out)
    assert pw.buffer == 0 and px.buffer == 1 and po.buffer == 1
    assert po.offset % 32 == 0 and po.offset >= px.offset + 4096 * 512 * 4
    # leafs first (weights first), then nodes
    assert [t.id for t in plan.tensors] == [w, x, out]


def test_tensor_io_validates_size():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    c = g.mul(a, b)
    g.mark_output(c)
    be = DummyBackend()
    plan = g.compile(be)
    with pytest.raises(FemlError):
        plan.write_tensor(be, a, bytes(7))
    with pytest.raises(FemlError):
        plan.read_tensor(be, a, bytearray(9))
    with pytest.raises(FemlError):
        plan.write_tensor(be, 10 ** 9, bytes(16))
    plan.write_tensor(be, a, np.arange(4, dtype=np.float32).tobytes())
    out = bytearray(16)
    plan.read_tensor(be, a, out)
    assert np.frombuffer(out, np.float32).tolist() == [0, 1, 2, 3]


def test_plan_release_frees_buffers():
    g = GraphBuilder()
    a = g.input("a", DType.F32, [4])
    b = g.input("b", DType.F32, [4])
    c = g.mul(a, b)
    g.mark_output(c)
    be = DummyBackend()
    plan = g.compile(be)
    assert len(be.buffers) == 1
    plan.release(be)
    assert be.buffers == {}


def test_uid_is_stable_fingerprint():
    def build():
        g = GraphBuilder()
        w = g.weight("w", DType.F32, [16, 8])
        x = g.input("x", DType.F32, [16, 32])
        g.mark_output(g.mul_mat(w, x))
        return g.compile(DummyBackend())
    p1, p2 = build(), build()
    assert p1.uid != 0 and p2.uid != 0
    assert p1.uid != p2.uid  # ids differ between graphs, as in the reference


# ---- registry / device (registry.rs:126-149) -------------------------------
class FakeRegistrar:
    def __init__(self, name, score, n=1):
        self._name, self._score, self._n = name, score, n

    def name(self):
        return self._name

    def device_count(self):
        return self._n

    def score(self):
        return self._score

    def device(self, i):
        reg = self

        class Dev:
            def init_backend(self):
                return reg._name
        return Dev()


def test_registry_open_best_by_score():
    r = F.Registry()
    r.register(FakeRegistrar("CPU", 100)).register(FakeRegistrar("B200x", 2000)).register(FakeRegistrar("none", 0))
    assert r.open_best() == "B200x"
    assert r.open("cpu", 0) == "CPU"
    with pytest.raises(FemlError):
        r.open("missing", 0)
    with pytest.raises(FemlError):
        F.Registry().open_best()


def test_b200_registrar_without_device_is_empty():
    reg = F.B200Registrar.probe()
    assert reg.name() == "B200"
    if reg.device_count() == 0:
        assert reg.score() == 0
        with pytest.raises(FemlError):
            F.B200Backend.open(0)


def test_rms_norm_builder():
    """graph.rs:140-142: unary, same shape and dtype as x; eps travels in
    op_params[0] as f32 bits; rms_norm may run in place (op.rs:98-110)."""
    import struct
    g = F.GraphBuilder()
    x = g.input("x", DType.F32, [4096, 3])
    r = g.rms_norm(x, 1e-5)
    w = g.weight("w", DType.Q8_0, [4096, 8])
    y = g.mul_mat(w, r)
    g.mark_output(y)
    plan = g.compile(DummyBackend())
    t = plan.find(r)
    assert t.op == Op.RMS_NORM and t.dtype == DType.F32 and t.shape[:2] == [4096, 3]
    assert t.op_params[0] == struct.unpack("<I", struct.pack("<f", 1e-5))[0]
    assert t.srcs == [plan.tensors.index(plan.find(x))]
    assert plan.find(y).srcs[1] == plan.tensors.index(t)
    assert F.B200Device(0).supports_op(Op.RMS_NORM, [DType.F32])
    assert not F.B200Device(0).supports_op(Op.RMS_NORM, [DType.F16])


def test_supports_op_matrix():
    dev = F.B200Device(0)
    for d in (DType.F32, DType.Q8_0, DType.Q4_0, DType.Q4_K):
        assert dev.supports_op(Op.MUL_MAT, [d, DType.F32])
        assert dev.supports_op(Op.MUL_MAT_ID, [d, DType.F32, DType.I32])
    assert not dev.supports_op(Op.MUL_MAT, [DType.Q8_0, DType.Q8_0])
    # Q5_K, Q6_K: mul_mat (decode GEMV) only
    for d in (DType.Q5_K, DType.Q6_K):
        assert dev.supports_op(Op.MUL_MAT, [d, DType.F32])
        assert not dev.supports_op(Op.MUL_MAT_ID, [d, DType.F32, DType.I32])
    assert not dev.supports_op(Op.MUL_MAT, [DType.Q3_K, DType.F32])
    assert not dev.supports_op(Op.MUL, [DType.F32, DType.F32])
    assert dev.supports_op(Op.RMS_NORM, [DType.F32])


# ---- C ABI ------------------------------------------------------------------
def test_library_exports_every_declared_symbol():
    from feml_b200 import _lib
    hdr = open(os.path.join(ROOT, "include", "feml_b200.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    declared = set(re.findall(r"\b((?:feml_b200|fb)_[a-z0-9_]+)\s*\(", hdr))
    assert len(declared) > 40
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, missing
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert declared <= bound, sorted(declared - bound)


def test_library_hides_internal_symbols():
    out = os.popen(f"nm -D --defined-only {F._L.LIB_PATH}").read()
    exported = [line.split()[-1] for line in out.splitlines() if " T " in line]
    assert all(s.startswith(("feml_b200_", "fb_")) for s in exported), exported


def test_mul_mat_launch_plans():
    """The host planner's launch counts (no GPU needed: 148 SMs assumed):
    the decode GEMV quantizes inside its one kernel; a GEMM is the activation
    quantizer plus the GEMM, plus a reduction when K is split (a tile grid
    that leaves most SMs idle) or when the last wave's overflow is split in K
    (19200 rows = 150 weight-row tiles: 2 past one wave); 258 tiles (11008 x
    512) take no tail split (the overflow is too wide to split)."""
    from feml_b200 import DType, ops
    assert ops.mul_mat_launches(DType.Q8_0, 4096, 4096, 1) == 1
    assert ops.mul_mat_launches(DType.Q4_0, 4096, 11008, 512) == 2
    assert ops.mul_mat_launches(DType.Q4_K, 14336, 4096, 64) == 3
    assert ops.mul_mat_launches(DType.Q8_0, 4096, 19200, 100) == 3
