"""feml_b200: a B200 (sm_100a) backend for feml's mul_mat / mul_mat_id path.

Python mirror of the feml-core API over the C ABI of libfeml_b200.so
(include/feml_b200.h). Names, argument meaning and error behaviour follow
the Rust crate feml-core:

    GraphBuilder  feml-core/src/graph.rs      (input, weight, view, mul_mat,
                                              mul_mat_id, mark_output, compile)
    GraphPlan     feml-core/src/plan.rs       (find, write_tensor, read_tensor,
                                              release)
    Backend       feml-core/src/backend.rs    (create_buffer, release_buffer,
                                              write, read, fill, synchronize,
                                              graph_compute, supports_op)
    Registry      feml-core/src/registry.rs   (register, open, open_best)

Build/compile/planning run in the C++ mirror inside the library; kernels run
on the GPU. There is no CPU execution path: B200Backend.open() fails on a
machine without an sm_100 device.
"""
import ctypes
from enum import IntEnum

from . import _lib as _L

__all__ = [
    "DType", "Op", "BufferUsage", "TensorFlags", "FemlError", "Backend", "B200Backend", "B200Device",
    "B200Registrar", "Registry", "GraphBuilder", "GraphPlan", "TensorMeta", "PlanTensor", "PlanBuffer",
    "layout_new", "layout_nbytes", "planner_plan", "version",
]


class DType(IntEnum):
    """feml-core/src/dtype.rs:14-35 (discriminant order is the ABI)."""
    I8 = 0
    I16 = 1
    I32 = 2
    I64 = 3
    F16 = 4
    F32 = 5
    F64 = 6
    Q4_0 = 7
    Q4_1 = 8
    Q5_0 = 9
    Q5_1 = 10
    Q8_0 = 11
    Q8_1 = 12
    Q2_K = 13
    Q3_K = 14
    Q4_K = 15
    Q5_K = 16
    Q6_K = 17
    Q8_K = 18

    def _traits(self):
        bs, ts, q = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int32()
        _check(_L.lib().fb_dtype_traits(int(self), ctypes.byref(bs), ctypes.byref(ts), ctypes.byref(q)))
        return bs.value, ts.value, bool(q.value)

    @property
    def block_size(self):
        return self._traits()[0]

    @property
    def type_size(self):
        return self._traits()[1]

    @property
    def is_quantized(self):
        return self._traits()[2]

    def row_size(self, n):
        bs, ts, _ = self._traits()
        if n % bs:
            raise FemlError("msg", f"{self.name.lower()}: row size {n} is not aligned to block size {bs}")
        return ts * n // bs


class Op(IntEnum):
    """feml-core/src/op.rs:12-43."""
    NONE = 0
    VIEW = 1
    MUL = 2
    ADD = 3
    MUL_MAT = 4
    MUL_MAT_ID = 5
    RMS_NORM = 6
    SOFTMAX = 7
    ROPE = 8
    SILU = 9
    GET_ROWS = 10
    CONCAT = 11
    COPY = 12
    DIAG_MASK_INF = 13
    SCALE = 14


class BufferUsage(IntEnum):
    """feml-core/src/backend.rs:52-57."""
    WEIGHTS = 0
    COMPUTE = 1


class TensorFlags:
    """feml-core/src/tensor.rs:48-68."""
    INPUT = 1
    OUTPUT = 2
    WEIGHT = 4


_KINDS = {1: "msg", 2: "unsupported", 3: "shape", 4: "backend", 5: "backend", 6: "backend"}


class FemlError(Exception):
    """feml-core/src/error.rs ErrorKind: kind in {msg, shape, unsupported, backend}."""

    def __init__(self, kind, message, code=None):
        super().__init__(message)
        self.kind = kind
        self.code = code


def _check(rc):
    if rc:
        msg = _L.lib().feml_b200_last_error().decode(errors="replace")
        raise FemlError(_KINDS.get(rc, "msg"), msg, rc)


def version():
    return _L.lib().feml_b200_version().decode()


def _dims(shape):
    shape = list(shape)
    arr = (ctypes.c_int64 * max(1, len(shape)))(*shape)
    return arr, len(shape)


# ---------------------------------------------------------------------------
# Backends
# ---------------------------------------------------------------------------
class Backend:
    """Python-side image of `trait Backend` (feml-core/src/backend.rs:86-122).

    Subclasses implemented in Python (test doubles such as the reference's
    DummyBackend) are driven by compile() through a C vtable."""

    def name(self):
        raise NotImplementedError

    def create_buffer(self, size, usage):
        raise NotImplementedError

    def release_buffer(self, handle):
        raise NotImplementedError

    def write(self, handle, offset, data):
        raise NotImplementedError

    def read(self, handle, offset, n):
        raise NotImplementedError

    def fill(self, handle, offset, value, length):
        raise NotImplementedError

    def synchronize(self):
        pass

    def graph_compute(self, plan):
        raise NotImplementedError

    def supports_op(self, op, src_dtypes):
        return False

    # -- adapter -------------------------------------------------------------
    def _vtable(self):
        if getattr(self, "_vt", None) is None:
            self._vt = _PyVTable(self)
        return self._vt


class _PyVTable:
    """ctypes callbacks that let the C++ compile() drive a Python backend."""

    def __init__(self, be):
        self.be = be
        self.exc = None
        self._name = None

        def guard(fn):
            def inner(*a):
                try:
                    r = fn(*a)
                    return 0 if r is None else r
                except Exception as e:  # noqa: BLE001 - re-raised after the C call
                    self.exc = e
                    return 1
            return inner

        def name(_):
            self._name = ctypes.create_string_buffer(self.be.name().encode())
            return ctypes.addressof(self._name)

        def create(_, size, usage, out):
            out[0] = int(self.be.create_buffer(int(size), BufferUsage(usage)))

        def release(_, h):
            self.be.release_buffer(int(h))

        def write(_, h, off, src, n):
            self.be.write(int(h), int(off), ctypes.string_at(src, n))

        def read(_, h, off, dst, n):
            data = self.be.read(int(h), int(off), int(n))
            ctypes.memmove(dst, bytes(data), n)

        def fill(_, h, off, v, n):
            self.be.fill(int(h), int(off), int(v), int(n))

        def sync(_):
            self.be.synchronize()

        def compute(_, plan):
            self.be.graph_compute(plan)

        def supports(_, op, dts, n):
            try:
                return 1 if self.be.supports_op(Op(op), [DType(dts[i]) for i in range(n)]) else 0
            except Exception as e:  # noqa: BLE001
                self.exc = e
                return 0

        self._cbs = (_L.NAME_FN(name), _L.CREATE_FN(guard(create)), _L.RELEASE_FN(guard(release)),
                     _L.WRITE_FN(guard(write)), _L.READ_FN(guard(read)), _L.FILL_FN(guard(fill)),
                     _L.SYNC_FN(guard(sync)), _L.COMPUTE_FN(guard(compute)), _L.SUPPORTS_FN(supports))
        self.vt = _L.VTable(None, *self._cbs)

    def ptr(self):
        return ctypes.byref(self.vt)

    def rethrow(self):
        if self.exc is not None:
            e, self.exc = self.exc, None
            raise e


class B200Backend(Backend):
    """The B200 execution stream: one device, one CUDA stream
    (BackendDevice::init_backend)."""

    def __init__(self, handle, device):
        self._h = handle
        self.device = device
        self._vt = None

    @classmethod
    def open(cls, device=0):
        h = ctypes.c_void_p()
        _check(_L.lib().feml_b200_open(int(device), ctypes.byref(h)))
        return cls(h, device)

    def close(self):
        if self._h:
            _L.lib().feml_b200_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def name(self):
        return _L.lib().feml_b200_name(self._h).decode()

    def create_buffer(self, size, usage=BufferUsage.COMPUTE):
        h = ctypes.c_uint32()
        _check(_L.lib().feml_b200_create_buffer(self._h, int(size), int(usage), ctypes.byref(h)))
        return h.value

    def release_buffer(self, handle):
        _check(_L.lib().feml_b200_release_buffer(self._h, int(handle)))

    def write(self, handle, offset, data):
        mv = memoryview(data).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer_copy(mv) if mv.readonly else (ctypes.c_char * len(mv)).from_buffer(mv)
        _check(_L.lib().feml_b200_write(self._h, int(handle), int(offset), buf, len(mv)))

    def write_ptr(self, handle, offset, host_ptr, n):
        _check(_L.lib().feml_b200_write(self._h, int(handle), int(offset), ctypes.c_void_p(host_ptr), int(n)))

    def read(self, handle, offset, n_or_out):
        if isinstance(n_or_out, int):
            out = bytearray(n_or_out)
        else:
            out = n_or_out
        mv = memoryview(out).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer(mv)
        _check(_L.lib().feml_b200_read(self._h, int(handle), int(offset), buf, len(mv)))
        return out

    def buffer_from_host_ptr(self, ptr, size, max_tensor_size):
        """A new Weights buffer holding `size` bytes copied to HBM straight
        from host memory at `ptr` (an int address, or any object exposing the
        buffer protocol); returns its handle."""
        if not isinstance(ptr, int):
            mv = memoryview(ptr).cast("B")
            if len(mv) < size:
                raise FemlError("msg", f"buffer_from_host_ptr: {len(mv)} bytes given, {size} requested")
            arr = (ctypes.c_char * len(mv)).from_buffer_copy(mv) if mv.readonly else \
                (ctypes.c_char * len(mv)).from_buffer(mv)
            ptr = ctypes.addressof(arr)
        h = ctypes.c_uint32()
        _check(_L.lib().feml_b200_buffer_from_host_ptr(self._h, ctypes.c_void_p(ptr), int(size), int(max_tensor_size),
                                                        ctypes.byref(h)))
        return h.value

    def read_ptr(self, handle, offset, host_ptr, n):
        _check(_L.lib().feml_b200_read(self._h, int(handle), int(offset), ctypes.c_void_p(host_ptr), int(n)))

    def fill(self, handle, offset, value, length):
        _check(_L.lib().feml_b200_fill(self._h, int(handle), int(offset), int(value), int(length)))

    def synchronize(self):
        _check(_L.lib().feml_b200_synchronize(self._h))

    def graph_compute(self, plan):
        p = plan._plan_ptr() if isinstance(plan, GraphPlan) else plan
        _check(_L.lib().feml_b200_graph_compute(self._h, p))

    def supports_op(self, op, src_dtypes):
        arr = (ctypes.c_int32 * max(1, len(src_dtypes)))(*[int(d) for d in src_dtypes])
        return bool(_L.lib().feml_b200_supports_op(self._h, int(op), arr, len(src_dtypes)))

    def device_ptr(self, handle):
        p, s = ctypes.c_void_p(), ctypes.c_uint64()
        _check(_L.lib().feml_b200_buffer_device_ptr(self._h, int(handle), ctypes.byref(p), ctypes.byref(s)))
        return p.value, s.value

    def stream(self):
        s = ctypes.c_void_p()
        _check(_L.lib().feml_b200_stream(self._h, ctypes.byref(s)))
        return s.value

    def scratch_bytes(self):
        v = ctypes.c_uint64()
        _check(_L.lib().feml_b200_scratch_bytes(self._h, ctypes.byref(v)))
        return v.value

    def set_plan_graphs(self, enable):
        """Replay CUDA graphs of repeated plans (default on)."""
        _check(_L.lib().feml_b200_set_plan_graphs(self._h, 1 if enable else 0))

    def plan_graphs(self):
        """(plans cached, plans replaying a graph)."""
        n, r = ctypes.c_int64(), ctypes.c_int64()
        _check(_L.lib().feml_b200_plan_graphs(self._h, ctypes.byref(n), ctypes.byref(r)))
        return n.value, r.value

    def plan_fused_nodes(self, plan):
        """Nodes of `plan` folded into a neighbouring kernel (rms_norm into a
        decode mul_mat, bias add / silu into a mul_mat's epilogue)."""
        n = ctypes.c_int64()
        _check(_L.lib().feml_b200_plan_fused_nodes(self._h, plan._plan_ptr(), ctypes.byref(n)))
        return n.value

    def device_allocations(self):
        """cudaMalloc calls this backend has made (buffers and scratch)."""
        v = ctypes.c_uint64()
        _check(_L.lib().feml_b200_device_allocations(self._h, ctypes.byref(v)))
        return v.value

    def reserve_scratch(self, n):
        _check(_L.lib().feml_b200_reserve_scratch(self._h, int(n)))

    def _vtable(self):
        if self._vt is None:
            vt = _L.VTable()
            _check(_L.lib().feml_b200_backend_vtable(self._h, ctypes.byref(vt)))
            self._vt = _NativeVTable(vt)
        return self._vt


class _NativeVTable:
    def __init__(self, vt):
        self.vt = vt

    def ptr(self):
        return ctypes.byref(self.vt)

    def rethrow(self):
        pass


class B200Device:
    """BackendDevice (feml-core/src/backend.rs:128-154) for one sm_100 GPU."""

    def __init__(self, index):
        self.index = index

    def info(self):
        di = _L.DeviceInfo()
        _check(_L.lib().feml_b200_device_info(self.index, ctypes.byref(di)))
        return {"name": di.name.decode(), "description": f"B200 device {self.index}",
                "memory_total": di.memory_total, "memory_free": di.memory_free,
                "compute_capability": (di.cc_major, di.cc_minor), "sm_count": di.sm_count,
                "device_type": "gpu", "caps": {"async_compute": bool(di.async_compute),
                                               "host_buffer": bool(di.host_buffer), "events": bool(di.events)}}

    def init_backend(self):
        return B200Backend.open(self.index)

    def supports_op(self, op, src_dtypes):
        arr = (ctypes.c_int32 * max(1, len(src_dtypes)))(*[int(d) for d in src_dtypes])
        return bool(_L.lib().feml_b200_supports_op(None, int(op), arr, len(src_dtypes)))

    def offload_op(self, op):
        return Op(op) in (Op.MUL_MAT, Op.MUL_MAT_ID)

    def buffer_from_host_ptr(self, ptr, size, max_tensor_size, backend=None):
        """BackendDevice::buffer_from_host_ptr (feml-core/src/backend.rs:145-153).
        Buffers here are owned by a backend (handles are backend-scoped), so
        the backend that will own the new Weights buffer is named here; see
        B200Backend.buffer_from_host_ptr."""
        if backend is None:
            raise FemlError("msg", "B200: buffer_from_host_ptr needs the backend that will own the buffer "
                                   "(buffer handles are backend-scoped)")
        return backend.buffer_from_host_ptr(ptr, size, max_tensor_size)


class B200Registrar:
    """BackendRegistrar (feml-core/src/backend.rs:157-165). Missing driver or
    devices give an empty registrar with score 0, never an error."""

    def __init__(self, count):
        self._count = count

    @classmethod
    def probe(cls):
        n = ctypes.c_int32()
        _check(_L.lib().feml_b200_device_count(ctypes.byref(n)))
        return cls(n.value)

    def name(self):
        return "B200"

    def device_count(self):
        return self._count

    def device(self, index):
        if not 0 <= index < self._count:
            raise FemlError("msg", f"B200: device {index} not found")
        return B200Device(index)

    def score(self):
        s = ctypes.c_uint32()
        _check(_L.lib().feml_b200_registrar_score(ctypes.byref(s)))
        return s.value if self._count else 0


class Registry:
    """feml-core/src/registry.rs: pluggable registrars, score-based choice."""

    def __init__(self):
        self._regs = []

    def register(self, registrar):
        self._regs.append(registrar)
        return self

    def registrars(self):
        return list(self._regs)

    def device_count(self):
        return sum(r.device_count() for r in self._regs)

    def find(self, name):
        for r in self._regs:
            if r.name().lower() == name.lower():
                return r
        return None

    def open(self, registrar_name, device_index):
        r = self.find(registrar_name)
        if r is None:
            raise FemlError("msg", f"backend registrar '{registrar_name}' not found")
        return r.device(device_index).init_backend()

    def open_best(self):
        best = None
        for r in self._regs:
            s = r.score()
            if s > 0 and r.device_count() > 0 and (best is None or s > best[0]):
                best = (s, r)
        if best is None:
            raise FemlError("msg", "no backend available")
        return best[1].device(0).init_backend()


# ---------------------------------------------------------------------------
# Graph building, compilation, plans
# ---------------------------------------------------------------------------
class TensorMeta:
    def __init__(self, id, dtype, shape, stride, flags, op):
        self.id, self.dtype, self.shape, self.stride, self.flags, self.op = id, dtype, shape, stride, flags, op

    def nbytes(self):
        return layout_nbytes(self.dtype, self.shape, self.stride)


class GraphBuilder:
    """feml-core/src/graph.rs GraphBuilder (C++ mirror in the library)."""

    def __init__(self):
        h = ctypes.c_void_p()
        _check(_L.lib().fb_graph_new(ctypes.byref(h)))
        self._h = h
        self._outputs = []

    def __del__(self):
        if getattr(self, "_h", None):
            _L.lib().fb_graph_free(self._h)
            self._h = None

    def _leaf(self, fn, name, dtype, shape):
        dims, rank = _dims(shape)
        out = ctypes.c_uint32()
        _check(fn(self._h, name.encode(), int(dtype), dims, rank, ctypes.byref(out)))
        return out.value

    def input(self, name, dtype, shape):
        return self._leaf(_L.lib().fb_graph_input, name, dtype, shape)

    def weight(self, name, dtype, shape):
        return self._leaf(_L.lib().fb_graph_weight, name, dtype, shape)

    def view(self, src, offset, shape):
        dims, rank = _dims(shape)
        out = ctypes.c_uint32()
        _check(_L.lib().fb_graph_view(self._h, int(src), int(offset), dims, rank, ctypes.byref(out)))
        return out.value

    def _bin(self, fn, a, b):
        out = ctypes.c_uint32()
        _check(fn(self._h, int(a), int(b), ctypes.byref(out)))
        return out.value

    def mul(self, a, b):
        return self._bin(_L.lib().fb_graph_mul, a, b)

    def add(self, a, b):
        return self._bin(_L.lib().fb_graph_add, a, b)

    def silu(self, x):
        out = ctypes.c_uint32()
        _check(_L.lib().fb_graph_silu(self._h, int(x), ctypes.byref(out)))
        return out.value

    def rms_norm(self, x, eps):
        """GraphBuilder::rms_norm (feml-core/src/graph.rs:140-142)."""
        out = ctypes.c_uint32()
        _check(_L.lib().fb_graph_rms_norm(self._h, int(x), float(eps), ctypes.byref(out)))
        return out.value

    def copy(self, x):
        out = ctypes.c_uint32()
        _check(_L.lib().fb_graph_copy(self._h, int(x), ctypes.byref(out)))
        return out.value

    def mul_mat(self, a, b):
        return self._bin(_L.lib().fb_graph_mul_mat, a, b)

    def mul_mat_id(self, weights, x, ids, n_selected):
        out = ctypes.c_uint32()
        _check(_L.lib().fb_graph_mul_mat_id(self._h, int(weights), int(x), int(ids), int(n_selected),
                                            ctypes.byref(out)))
        return out.value

    def mark_output(self, t):
        _check(_L.lib().fb_graph_mark_output(self._h, int(t)))
        self._outputs.append(t)

    def outputs(self):
        return list(self._outputs)

    def tensor(self, t):
        dt, fl, op = ctypes.c_int32(), ctypes.c_uint32(), ctypes.c_int32()
        ne, nb = (ctypes.c_int64 * 4)(), (ctypes.c_uint64 * 4)()
        try:
            _check(_L.lib().fb_graph_tensor_info(self._h, int(t), ctypes.byref(dt), ne, nb, ctypes.byref(fl),
                                                 ctypes.byref(op)))
        except FemlError:
            return None
        return TensorMeta(t, DType(dt.value), list(ne), list(nb), fl.value, Op(op.value))

    def compile(self, backend):
        vt = backend._vtable()
        p = ctypes.c_void_p()
        rc = _L.lib().fb_graph_compile(self._h, vt.ptr(), ctypes.byref(p))
        vt.rethrow()
        _check(rc)
        return GraphPlan(p, vt)


class PlanTensor:
    def __init__(self, pt):
        self.id = pt.id
        self.op = Op(pt.op)
        self.op_params = list(pt.op_params)
        self.srcs = [pt.srcs[i] for i in range(pt.n_srcs)]
        self.buffer = pt.buffer
        self.offset = pt.offset
        self.dtype = DType(pt.dtype)
        self.flags = pt.flags
        self.shape = list(pt.ne)
        self.stride = list(pt.nb)

    def nbytes(self):
        return layout_nbytes(self.dtype, self.shape, self.stride)


class PlanBuffer:
    def __init__(self, pb):
        self.handle, self.size, self.usage = pb.handle, pb.size, BufferUsage(pb.usage)


class GraphPlan:
    """feml-core/src/plan.rs GraphPlan (owned by the C++ mirror)."""

    def __init__(self, handle, vt):
        self._h = handle
        self._vt = vt
        p = _L.lib().fb_plan_get(handle).contents
        self.uid = p.uid
        self.tensors = [PlanTensor(p.tensors[i]) for i in range(p.n_tensors)]
        self.nodes = [p.nodes[i] for i in range(p.n_nodes)]
        self.buffers = [PlanBuffer(p.buffers[i]) for i in range(p.n_buffers)]

    def __del__(self):
        if getattr(self, "_h", None):
            _L.lib().fb_plan_free(self._h)
            self._h = None

    def _plan_ptr(self):
        return _L.lib().fb_plan_get(self._h)

    def find(self, tensor_id):
        i = _L.lib().fb_plan_find(self._h, int(tensor_id))
        return None if i < 0 else self.tensors[i]

    def write_tensor(self, backend, tensor_id, data):
        mv = memoryview(data).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer_copy(mv) if mv.readonly else (ctypes.c_char * len(mv)).from_buffer(mv)
        vt = backend._vtable()
        rc = _L.lib().fb_plan_write_tensor(self._h, vt.ptr(), int(tensor_id), buf, len(mv))
        vt.rethrow()
        _check(rc)

    def read_tensor(self, backend, tensor_id, out):
        mv = memoryview(out).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer(mv)
        vt = backend._vtable()
        rc = _L.lib().fb_plan_read_tensor(self._h, vt.ptr(), int(tensor_id), buf, len(mv))
        vt.rethrow()
        _check(rc)
        return out

    def release(self, backend):
        vt = backend._vtable()
        rc = _L.lib().fb_plan_release(self._h, vt.ptr())
        vt.rethrow()
        _check(rc)


def layout_new(dtype, shape):
    """Layout::new (feml-core/src/layout.rs:32-48): ggml byte strides."""
    dims, rank = _dims(shape)
    nb = (ctypes.c_uint64 * 4)()
    _check(_L.lib().fb_layout_new(int(dtype), dims, rank, nb))
    return list(nb)


def layout_nbytes(dtype, shape, stride):
    """Layout::nbytes (feml-core/src/layout.rs:51-60)."""
    ne = list(shape) + [1] * (4 - len(shape))
    ne_a = (ctypes.c_int64 * 4)(*ne)
    nb_a = (ctypes.c_uint64 * 4)(*stride)
    out = ctypes.c_uint64()
    _check(_L.lib().fb_layout_nbytes(int(dtype), ne_a, nb_a, ctypes.byref(out)))
    return out.value


def planner_plan(tensors, order):
    """Run the memory planner (feml-core/src/planner.rs:156-261) on tensor
    descriptions: dicts with id, dtype, shape, flags, op, srcs (ids),
    view_src (id or 0), view_offset. Returns ({id: (kind, offset)},
    weights_size, compute_size) with kind 0 = Weights, 1 = Compute."""
    arr = (_L.PlannerTensor * max(1, len(tensors)))()
    for i, t in enumerate(tensors):
        shape = list(t["shape"])
        arr[i].id = t["id"]
        arr[i].dtype = int(t.get("dtype", DType.F32))
        for j in range(4):
            arr[i].ne[j] = shape[j] if j < len(shape) else 1
        arr[i].rank = len(shape)
        arr[i].flags = t.get("flags", 0)
        arr[i].op = int(t.get("op", Op.NONE))
        srcs = t.get("srcs", [])
        arr[i].n_srcs = len(srcs)
        for j, s in enumerate(srcs):
            arr[i].srcs[j] = s
        arr[i].view_src = t.get("view_src", 0)
        arr[i].view_offset = t.get("view_offset", 0)
    order_a = (ctypes.c_int64 * max(1, len(order)))(*order)
    kinds = (ctypes.c_int32 * max(1, len(tensors)))()
    offs = (ctypes.c_uint64 * max(1, len(tensors)))()
    ws, cs = ctypes.c_uint64(), ctypes.c_uint64()
    _check(_L.lib().fb_planner_plan(arr, len(tensors), order_a, len(order), kinds, offs, ctypes.byref(ws),
                                    ctypes.byref(cs)))
    return ({t["id"]: (kinds[i], offs[i]) for i, t in enumerate(tensors)}, ws.value, cs.value)
