"""Loads libfeml_b200.so and declares its C signatures (include/feml_b200.h).

The library is built in-tree by feml_b200/build.py. There is no fallback:
importing the package without the built library raises ImportError.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfeml_b200.so")

c_int, c_i32, c_u32, c_i64, c_u64, c_u8 = (ctypes.c_int, ctypes.c_int32, ctypes.c_uint32,
                                          ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint8)
vp = ctypes.c_void_p
cp = ctypes.c_char_p

FB_MAX_SRC = 4


class PlanTensor(ctypes.Structure):
    _fields_ = [("id", c_u32), ("op", c_i32), ("op_params", c_u32 * 2), ("n_srcs", c_i32),
                ("srcs", c_i32 * FB_MAX_SRC), ("buffer", c_i32), ("offset", c_u64), ("dtype", c_i32),
                ("flags", c_u32), ("ne", c_i64 * 4), ("nb", c_u64 * 4)]


class PlanBuffer(ctypes.Structure):
    _fields_ = [("handle", c_u32), ("size", c_u64), ("usage", c_i32)]


class Plan(ctypes.Structure):
    _fields_ = [("uid", c_u64), ("tensors", ctypes.POINTER(PlanTensor)), ("n_tensors", c_i64),
                ("nodes", ctypes.POINTER(c_i64)), ("n_nodes", c_i64),
                ("buffers", ctypes.POINTER(PlanBuffer)), ("n_buffers", c_i64)]


NAME_FN = ctypes.CFUNCTYPE(vp, vp)  # returns a char* kept alive by the caller
CREATE_FN = ctypes.CFUNCTYPE(c_int, vp, c_u64, c_i32, ctypes.POINTER(c_u32))
RELEASE_FN = ctypes.CFUNCTYPE(c_int, vp, c_u32)
WRITE_FN = ctypes.CFUNCTYPE(c_int, vp, c_u32, c_u64, vp, c_u64)
READ_FN = ctypes.CFUNCTYPE(c_int, vp, c_u32, c_u64, vp, c_u64)
FILL_FN = ctypes.CFUNCTYPE(c_int, vp, c_u32, c_u64, c_u8, c_u64)
SYNC_FN = ctypes.CFUNCTYPE(c_int, vp)
COMPUTE_FN = ctypes.CFUNCTYPE(c_int, vp, ctypes.POINTER(Plan))
SUPPORTS_FN = ctypes.CFUNCTYPE(c_int, vp, c_i32, ctypes.POINTER(c_i32), c_i32)
PREPARE_FN = ctypes.CFUNCTYPE(c_int, vp, ctypes.POINTER(Plan))


class VTable(ctypes.Structure):
    _fields_ = [("ctx", vp), ("name", NAME_FN), ("create_buffer", CREATE_FN), ("release_buffer", RELEASE_FN),
                ("write", WRITE_FN), ("read", READ_FN), ("fill", FILL_FN), ("synchronize", SYNC_FN),
                ("graph_compute", COMPUTE_FN), ("supports_op", SUPPORTS_FN), ("prepare_plan", PREPARE_FN)]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("memory_total", c_u64), ("memory_free", c_u64),
                ("cc_major", c_i32), ("cc_minor", c_i32), ("sm_count", c_i32), ("device_type", c_i32),
                ("async_compute", c_i32), ("host_buffer", c_i32), ("events", c_i32)]


class PlannerTensor(ctypes.Structure):
    _fields_ = [("id", c_u32), ("dtype", c_i32), ("ne", c_i64 * 4), ("rank", c_i32), ("flags", c_u32),
                ("op", c_i32), ("n_srcs", c_i32), ("srcs", c_u32 * FB_MAX_SRC), ("view_src", c_u32),
                ("view_offset", c_u64)]


class GgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("dtype", c_i32), ("ggml_type", c_u32), ("n_dims", c_i32),
                ("ne", c_i64 * 4), ("offset", c_u64), ("nbytes", c_u64)]


# (name, restype, argtypes) for every exported symbol in include/feml_b200.h
SIGNATURES = [
    ("feml_b200_last_error", cp, []),
    ("feml_b200_version", cp, []),
    ("feml_b200_device_count", c_int, [ctypes.POINTER(c_i32)]),
    ("feml_b200_registrar_score", c_int, [ctypes.POINTER(c_u32)]),
    ("feml_b200_device_info", c_int, [c_i32, ctypes.POINTER(DeviceInfo)]),
    ("feml_b200_open", c_int, [c_i32, ctypes.POINTER(vp)]),
    ("feml_b200_close", c_int, [vp]),
    ("feml_b200_name", cp, [vp]),
    ("feml_b200_create_buffer", c_int, [vp, c_u64, c_i32, ctypes.POINTER(c_u32)]),
    ("feml_b200_release_buffer", c_int, [vp, c_u32]),
    ("feml_b200_write", c_int, [vp, c_u32, c_u64, vp, c_u64]),
    ("feml_b200_read", c_int, [vp, c_u32, c_u64, vp, c_u64]),
    ("feml_b200_fill", c_int, [vp, c_u32, c_u64, c_u8, c_u64]),
    ("feml_b200_synchronize", c_int, [vp]),
    ("feml_b200_supports_op", c_int, [vp, c_i32, ctypes.POINTER(c_i32), c_i32]),
    ("feml_b200_graph_compute", c_int, [vp, ctypes.POINTER(Plan)]),
    ("feml_b200_prepare_plan", c_int, [vp, ctypes.POINTER(Plan)]),
    ("feml_b200_plan_fused_nodes", c_int, [vp, ctypes.POINTER(Plan), ctypes.POINTER(c_i64)]),
    ("feml_b200_backend_vtable", c_int, [vp, ctypes.POINTER(VTable)]),
    ("feml_b200_buffer_device_ptr", c_int, [vp, c_u32, ctypes.POINTER(vp), ctypes.POINTER(c_u64)]),
    ("feml_b200_stream", c_int, [vp, ctypes.POINTER(vp)]),
    ("feml_b200_scratch_bytes", c_int, [vp, ctypes.POINTER(c_u64)]),
    ("feml_b200_reserve_scratch", c_int, [vp, c_u64]),
    ("feml_b200_device_allocations", c_int, [vp, ctypes.POINTER(c_u64)]),
    ("feml_b200_set_plan_graphs", c_int, [vp, c_i32]),
    ("feml_b200_plan_graphs", c_int, [vp, ctypes.POINTER(c_i64), ctypes.POINTER(c_i64)]),
    ("fb_graph_new", c_int, [ctypes.POINTER(vp)]),
    ("fb_graph_free", None, [vp]),
    ("fb_graph_input", c_int, [vp, cp, c_i32, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_u32)]),
    ("fb_graph_weight", c_int, [vp, cp, c_i32, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_u32)]),
    ("fb_graph_view", c_int, [vp, c_u32, c_u64, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_u32)]),
    ("fb_graph_mul", c_int, [vp, c_u32, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_add", c_int, [vp, c_u32, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_silu", c_int, [vp, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_rms_norm", c_int, [vp, c_u32, ctypes.c_float, ctypes.POINTER(c_u32)]),
    ("fb_graph_copy", c_int, [vp, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_mul_mat", c_int, [vp, c_u32, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_mul_mat_id", c_int, [vp, c_u32, c_u32, c_u32, c_u32, ctypes.POINTER(c_u32)]),
    ("fb_graph_mark_output", c_int, [vp, c_u32]),
    ("fb_graph_tensor_info", c_int, [vp, c_u32, ctypes.POINTER(c_i32), ctypes.POINTER(c_i64),
                                     ctypes.POINTER(c_u64), ctypes.POINTER(c_u32), ctypes.POINTER(c_i32)]),
    ("fb_graph_compile", c_int, [vp, ctypes.POINTER(VTable), ctypes.POINTER(vp)]),
    ("fb_plan_get", ctypes.POINTER(Plan), [vp]),
    ("fb_plan_find", c_i64, [vp, c_u32]),
    ("fb_plan_write_tensor", c_int, [vp, ctypes.POINTER(VTable), c_u32, vp, c_u64]),
    ("fb_plan_read_tensor", c_int, [vp, ctypes.POINTER(VTable), c_u32, vp, c_u64]),
    ("fb_plan_release", c_int, [vp, ctypes.POINTER(VTable)]),
    ("fb_plan_free", None, [vp]),
    ("fb_planner_plan", c_int, [ctypes.POINTER(PlannerTensor), c_i64, ctypes.POINTER(c_i64), c_i64,
                                ctypes.POINTER(c_i32), ctypes.POINTER(c_u64), ctypes.POINTER(c_u64),
                                ctypes.POINTER(c_u64)]),
    ("fb_layout_new", c_int, [c_i32, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_u64)]),
    ("fb_layout_nbytes", c_int, [c_i32, ctypes.POINTER(c_i64), ctypes.POINTER(c_u64), ctypes.POINTER(c_u64)]),
    ("fb_dtype_traits", c_int, [c_i32, ctypes.POINTER(c_i64), ctypes.POINTER(c_i64), ctypes.POINTER(c_i32)]),
    ("feml_b200_quantize", c_int, [c_i32, vp, c_u64, vp, c_i64, c_i64, vp]),
    ("feml_b200_mul_mat_workspace", c_int, [c_i32, c_i64, c_i64, c_i64, ctypes.POINTER(c_u64)]),
    ("feml_b200_mul_mat", c_int, [c_i32, vp, c_u64, vp, c_u64, vp, c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp]),
    ("feml_b200_mul_mat_launches", c_int, [c_i32, c_i64, c_i64, c_i64, ctypes.POINTER(c_i32)]),
    ("feml_b200_mul_mat_noalloc", c_int, [c_i32, vp, c_u64, vp, c_u64, vp, c_u64, c_i64, c_i64, c_i64, vp]),
    ("feml_b200_mul_mat_noalloc_limit", c_u64, []),
    ("feml_b200_mul_mat_id_workspace", c_int, [c_i32, c_i64, c_i64, c_i64, c_i64, c_i64, ctypes.POINTER(c_u64)]),
    ("feml_b200_mul_mat_id", c_int, [c_i32, vp, c_u64, c_u64, c_i64, vp, c_u64, vp, c_u64, c_i64, vp, c_u64,
                                     c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp, vp]),
    ("feml_b200_mul_mat_peer", c_int, [c_i32, vp, c_u64, vp, c_u64, vp, vp, vp, c_i32, c_u64, vp, vp, c_i64, c_i64,
                                       c_i64, vp, vp]),
    ("feml_b200_peer_wait", c_int, [vp, vp, c_i32, vp, vp]),
    ("feml_b200_peer_wait_timeout", c_int, [vp, vp, c_i32, c_u64, vp, vp]),
    ("feml_b200_mul_mat_id_peer", c_int, [c_i32, vp, c_u64, c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp, c_u64, c_i64,
                                          vp, vp, vp, c_i32, c_u64, c_u64, vp, vp, c_i64, c_i64, c_i64, vp, c_u64, vp,
                                          vp]),
    ("feml_b200_mul_mat_id_peer_owned", c_int, [c_i32, vp, c_u64, c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp, c_u64,
                                                c_i64, vp, vp, vp, c_i32, c_u64, c_u64, c_i64, vp, vp, c_i64, c_i64,
                                                c_i64, vp, c_u64, vp, vp]),
    ("feml_b200_ipc_open", c_int, [vp, c_u64, ctypes.POINTER(vp)]),
    ("feml_b200_ipc_close", c_int, [vp]),
    ("feml_b200_ipc_export", c_int, [vp, vp, c_u64, ctypes.POINTER(c_u64)]),
    ("feml_b200_mul_mat_id_shard", c_int, [c_i32, vp, c_u64, c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp, c_u64, c_i64,
                                           vp, c_u64, c_u64, c_i64, c_i64, c_i64, vp, c_u64, vp, vp]),
    ("feml_b200_moe_route", c_int, [vp, c_u64, c_i64, c_i64, c_i64, vp, vp, vp, vp, vp]),
    ("feml_b200_block_dots", c_int, [c_i32, vp, c_u64, vp, c_i64, c_i64, c_i64, vp, vp]),
    ("feml_b200_buffer_from_host_ptr", c_int, [vp, vp, c_u64, c_u64, ctypes.POINTER(c_u32)]),
    ("feml_b200_gguf_open", c_int, [cp, ctypes.POINTER(vp)]),
    ("feml_b200_gguf_close", c_int, [vp]),
    ("feml_b200_gguf_info", c_int, [vp, ctypes.POINTER(c_u32), ctypes.POINTER(c_u64), ctypes.POINTER(c_u64),
                                    ctypes.POINTER(c_i64), ctypes.POINTER(c_i64)]),
    ("feml_b200_gguf_tensor", c_int, [vp, c_i64, ctypes.POINTER(GgufTensor)]),
    ("feml_b200_gguf_find_tensor", c_int, [vp, cp, ctypes.POINTER(c_i64)]),
    ("feml_b200_gguf_tensor_data", c_int, [vp, c_i64, ctypes.POINTER(vp)]),
    ("feml_b200_gguf_kv", c_int, [vp, c_i64, ctypes.POINTER(cp), ctypes.POINTER(c_u32), ctypes.POINTER(c_u32),
                                  ctypes.POINTER(c_u64)]),
    ("feml_b200_gguf_find_kv", c_int, [vp, cp, ctypes.POINTER(c_i64)]),
    ("feml_b200_gguf_kv_int", c_int, [vp, c_i64, ctypes.POINTER(c_i64)]),
    ("feml_b200_gguf_kv_float", c_int, [vp, c_i64, ctypes.POINTER(ctypes.c_double)]),
    ("feml_b200_gguf_kv_str", c_int, [vp, c_i64, c_i64, ctypes.POINTER(vp), ctypes.POINTER(c_u64)]),
    ("feml_b200_gguf_kv_array_data", c_int, [vp, c_i64, ctypes.POINTER(vp)]),
]

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"feml_b200: {LIB_PATH} is missing; build it with `python feml_b200/build.py` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib
