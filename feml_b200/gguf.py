"""GGUF model files through the library's reader (feml_b200_gguf_*).

GGUF is the llama.cpp / ggml model container that feml's roadmap names as the
source of quantized weights (docs/DESIGN.md:282-286 of the reference: mmap +
`buffer_from_host_ptr`). The file is mapped read-only by the C++ reader;
tensor bytes are exposed as read-only numpy views of the mapping and go to
the device in one copy each, either into a compiled plan's weight tensor
(`write_to_plan`) or as one Weights buffer holding the whole data section
(`upload`).

    with GGUFFile(path) as f:
        f.metadata["general.architecture"]
        info = f.tensor("blk.0.ffn_down.weight")   # dtype, shape (ggml ne order)
        f.write_to_plan(plan, backend, tensor_id, info.name)
"""
import ctypes
from typing import NamedTuple, Optional, Tuple

import numpy as np

from . import DType, FemlError, _check
from . import _lib as _L

# GGUF metadata value types (public specification)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_NUMPY = {U8: np.uint8, I8: np.int8, U16: np.uint16, I16: np.int16, U32: np.uint32, I32: np.int32,
          F32: np.float32, BOOL: np.bool_, U64: np.uint64, I64: np.int64, F64: np.float64}


class GGUFTensorInfo(NamedTuple):
    name: str
    dtype: Optional[DType]   # None when feml has no counterpart (BF16, IQ types ...)
    ggml_type: int
    shape: Tuple[int, ...]   # ggml ne order, ne[0] contiguous
    offset: int              # from the start of the file
    nbytes: int


class GGUFFile:
    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(_L.lib().feml_b200_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h
        ver, al, doff = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint64()
        nkv, nt = ctypes.c_int64(), ctypes.c_int64()
        _check(_L.lib().feml_b200_gguf_info(h, ctypes.byref(ver), ctypes.byref(al), ctypes.byref(doff),
                                            ctypes.byref(nkv), ctypes.byref(nt)))
        self.version, self.alignment, self.data_offset = ver.value, al.value, doff.value
        self._n_kv, self._n_tensors = nkv.value, nt.value
        self._metadata = None
        self._tensors = None

    # ---- lifetime ----------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            _L.lib().feml_b200_gguf_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()

    def _live(self):
        if not self._h:
            raise FemlError("msg", "gguf: file is closed")
        return self._h

    # ---- metadata ----------------------------------------------------------
    def _value(self, i, typ, elem, count):
        h, L = self._live(), _L.lib()
        if typ == STRING:
            s, n = ctypes.c_void_p(), ctypes.c_uint64()
            _check(L.feml_b200_gguf_kv_str(h, i, 0, ctypes.byref(s), ctypes.byref(n)))
            return ctypes.string_at(s.value, n.value).decode("utf-8", errors="replace") if n.value else ""
        if typ == ARRAY:
            if elem == STRING:
                out = []
                s, n = ctypes.c_void_p(), ctypes.c_uint64()
                for j in range(count):
                    _check(L.feml_b200_gguf_kv_str(h, i, j, ctypes.byref(s), ctypes.byref(n)))
                    out.append(ctypes.string_at(s.value, n.value).decode("utf-8", errors="replace")
                               if n.value else "")
                return out
            p = ctypes.c_void_p()
            _check(L.feml_b200_gguf_kv_array_data(h, i, ctypes.byref(p)))
            dt = np.dtype(_NUMPY[elem])
            if count == 0:
                return np.zeros(0, dtype=dt)
            raw = ctypes.string_at(p.value, count * dt.itemsize)
            return np.frombuffer(raw, dtype=dt.newbyteorder("<")).astype(dt)
        if typ in (F32, F64):
            v = ctypes.c_double()
            _check(L.feml_b200_gguf_kv_float(h, i, ctypes.byref(v)))
            return v.value
        v = ctypes.c_int64()
        _check(L.feml_b200_gguf_kv_int(h, i, ctypes.byref(v)))
        return bool(v.value) if typ == BOOL else v.value

    @property
    def metadata(self):
        """Key -> value: ints, floats, bools, strings; numeric arrays as numpy
        arrays, string arrays as lists."""
        if self._metadata is None:
            h, L = self._live(), _L.lib()
            md = {}
            for i in range(self._n_kv):
                key, typ, elem, cnt = ctypes.c_char_p(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint64()
                _check(L.feml_b200_gguf_kv(h, i, ctypes.byref(key), ctypes.byref(typ), ctypes.byref(elem),
                                           ctypes.byref(cnt)))
                md[key.value.decode("utf-8", errors="replace")] = self._value(i, typ.value, elem.value, cnt.value)
            self._metadata = md
        return self._metadata

    # ---- tensors -----------------------------------------------------------
    @property
    def tensors(self):
        if self._tensors is None:
            h, L = self._live(), _L.lib()
            out = []
            t = _L.GgufTensor()
            for i in range(self._n_tensors):
                _check(L.feml_b200_gguf_tensor(h, i, ctypes.byref(t)))
                # names that are not UTF-8 keep their bytes (surrogate escapes), so
                # they can be looked up again
                out.append(GGUFTensorInfo(t.name.decode("utf-8", errors="surrogateescape"),
                                          DType(t.dtype) if t.dtype >= 0 else None, t.ggml_type,
                                          tuple(t.ne[d] for d in range(t.n_dims)), t.offset, t.nbytes))
            self._tensors = out
        return self._tensors

    def _index(self, name):
        i = ctypes.c_int64()
        _check(_L.lib().feml_b200_gguf_find_tensor(self._live(), name.encode("utf-8", errors="surrogateescape"),
                                                   ctypes.byref(i)))
        return i.value

    def tensor(self, name):
        return self.tensors[self._index(name)]

    def tensor_bytes(self, name):
        """Read-only uint8 view of the tensor's bytes in the mapping (valid
        while the file is open)."""
        i = self._index(name)
        info = self.tensors[i]
        if info.nbytes == 0:
            raise FemlError("unsupported", f"gguf: tensor '{name}' has a type of unknown size ({info.ggml_type})")
        p = ctypes.c_void_p()
        _check(_L.lib().feml_b200_gguf_tensor_data(self._live(), i, ctypes.byref(p)))
        arr = np.ctypeslib.as_array((ctypes.c_uint8 * info.nbytes).from_address(p.value))
        arr.flags.writeable = False
        return arr

    # ---- upload --------------------------------------------------------------
    def write_to_plan(self, plan, backend, tensor_id, name):
        """Copy tensor `name` into the plan's tensor `tensor_id` (dtype and
        shape must match; the copy goes straight from the mapping)."""
        info = self.tensor(name)
        pt = plan.find(tensor_id)
        if pt is None:
            raise FemlError("msg", f"gguf: tensor id {tensor_id} is not in the plan")
        if info.dtype is None or int(info.dtype) != int(pt.dtype):
            raise FemlError("shape", f"gguf: '{name}' is {info.dtype}, the plan tensor is {DType(pt.dtype)}")
        ne = [int(v) for v in pt.shape]
        if tuple(ne[:len(info.shape)]) != info.shape or any(v != 1 for v in ne[len(info.shape):]):
            raise FemlError("shape", f"gguf: '{name}' has shape {info.shape}, the plan tensor {tuple(ne)}")
        p = ctypes.c_void_p()
        _check(_L.lib().feml_b200_gguf_tensor_data(self._live(), self._index(name), ctypes.byref(p)))
        vt = backend._vtable()
        rc = _L.lib().fb_plan_write_tensor(plan._h, vt.ptr(), int(tensor_id), p, info.nbytes)
        vt.rethrow()
        _check(rc)

    def upload(self, backend):
        """One Weights buffer holding the whole data section, copied once from
        the mapping (BackendDevice::buffer_from_host_ptr); returns (handle,
        {name: byte offset of the tensor inside the buffer})."""
        sized = [t for t in self.tensors if t.nbytes]
        if not sized:
            raise FemlError("msg", "gguf: no tensors of known size")
        end = max(t.offset + t.nbytes for t in sized)
        first = self.tensors[0].offset if self.tensors else self.data_offset
        p = ctypes.c_void_p()
        _check(_L.lib().feml_b200_gguf_tensor_data(self._live(), 0, ctypes.byref(p)))
        base = p.value - (first - self.data_offset)
        size = end - self.data_offset
        handle = backend.buffer_from_host_ptr(base, size, max(t.nbytes for t in sized))
        return handle, {t.name: t.offset - self.data_offset for t in self.tensors}
