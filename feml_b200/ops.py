"""Kernel-level entry points of libfeml_b200.so on torch CUDA tensors.

torch only provides device memory and the current stream here; every op
runs a kernel of this library (include/feml_b200.h, section 3).
Layouts follow ggml: a weight matrix ne=[K, M] is a uint8 tensor [M, row_bytes];
activations ne=[K, N] are f32 [N, K]; results ne=[M, N] are f32 [N, M].
"""
import ctypes

import torch

from . import DType, FemlError, _check
from . import _lib as _L


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def row_bytes(dtype, k):
    return DType(dtype).row_size(k)


def quantize(dtype, x):
    """Quantize f32 rows [rows, k] -> uint8 [rows, row_bytes] (ggml blocks)."""
    assert x.is_cuda and x.dtype == torch.float32 and x.dim() == 2
    rows, k = x.shape
    out = torch.empty((rows, row_bytes(dtype, k)), dtype=torch.uint8, device=x.device)
    _check(_L.lib().feml_b200_quantize(int(dtype), _ptr(x), x.stride(0) * 4, _ptr(out), rows, k, _stream()))
    return out


def mul_mat_workspace(wtype, K, M, N):
    v = ctypes.c_uint64()
    _check(_L.lib().feml_b200_mul_mat_workspace(int(wtype), K, M, N, ctypes.byref(v)))
    return v.value


def mul_mat_launches(wtype, K, M, N):
    """Kernel launches one mul_mat of this shape enqueues."""
    v = ctypes.c_int32()
    _check(_L.lib().feml_b200_mul_mat_launches(int(wtype), K, M, N, ctypes.byref(v)))
    return v.value


def mul_mat(wtype, w, x, K, out=None, workspace=None):
    """w: uint8 [M, row_bytes] (or f32 [M, K] for F32); x: f32 [N, K] -> f32 [N, M]."""
    M = w.shape[0]
    N = x.shape[0]
    w_nb1 = w.stride(0) * w.element_size()
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=x.device)
    need = mul_mat_workspace(wtype, K, M, N)
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    ws_ptr = _ptr(workspace) if workspace is not None else ctypes.c_void_p()
    ws_n = workspace.numel() if workspace is not None else 0
    _check(_L.lib().feml_b200_mul_mat(int(wtype), _ptr(w), w_nb1, _ptr(x), x.stride(0) * 4, _ptr(out),
                                      out.stride(0) * 4, K, M, N, ws_ptr, ws_n, _stream()))
    return out


def mul_mat_noalloc(wtype, w, x, K, out):
    """feml_b200_mul_mat_noalloc: mul_mat with the library's fixed device
    scratch (no workspace, no allocation inside the call); `out` is given."""
    M, N = w.shape[0], x.shape[0]
    _check(_L.lib().feml_b200_mul_mat_noalloc(int(wtype), _ptr(w), w.stride(0) * w.element_size(), _ptr(x),
                                              x.stride(0) * 4, _ptr(out), out.stride(0) * 4, K, M, N, _stream()))
    return out


def mul_mat_noalloc_limit():
    return int(_L.lib().feml_b200_mul_mat_noalloc_limit())


def mul_mat_id_workspace(wtype, K, M, N, n_selected, n_experts):
    v = ctypes.c_uint64()
    _check(_L.lib().feml_b200_mul_mat_id_workspace(int(wtype), K, M, N, n_selected, n_experts, ctypes.byref(v)))
    return v.value


def mul_mat_id(wtype, w, x, ids, K, out=None, workspace=None, status=None):
    """w: uint8 [E, M, row_bytes] (or f32 [E, M, K]); x: f32 [N, K];
    ids: int32 [N, n_sel] -> f32 [N, n_sel, M] (ggml dst ne=[M, n_sel, N])."""
    E, M = w.shape[0], w.shape[1]
    N, n_sel = ids.shape
    es = w.element_size()
    if out is None:
        out = torch.empty((N, n_sel, M), dtype=torch.float32, device=x.device)
    need = mul_mat_id_workspace(wtype, K, M, N, n_sel, E)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    _check(_L.lib().feml_b200_mul_mat_id(int(wtype), _ptr(w), w.stride(1) * es, w.stride(0) * es, E, _ptr(x),
                                         x.stride(0) * 4, _ptr(ids), ids.stride(0) * 4, n_sel, _ptr(out),
                                         out.stride(1) * 4, out.stride(0) * 4, K, M, N, _ptr(workspace),
                                         workspace.numel(), st, _stream()))
    return out


def local_experts(n_experts, shard, n_shards):
    """Experts owned by `shard` when expert e lives on shard e % n_shards."""
    return max(0, (n_experts - shard + n_shards - 1) // n_shards)


def mul_mat_id_shard(wtype, w_local, x, ids, K, n_experts, shard, n_shards, out, workspace=None, status=None):
    """Expert-sharded mul_mat_id: w_local holds the experts e with
    e % n_shards == shard (local index e // n_shards). Writes only the
    out[t, s, :] slots routed to those experts (invalid ids: zeros + status)."""
    E_loc, M = w_local.shape[0], w_local.shape[1]
    if E_loc != local_experts(n_experts, shard, n_shards):
        raise FemlError("msg", f"mul_mat_id_shard: shard {shard}/{n_shards} of {n_experts} experts holds "
                               f"{local_experts(n_experts, shard, n_shards)} experts, got {E_loc}")
    N, n_sel = ids.shape
    es = w_local.element_size()
    need = mul_mat_id_workspace(wtype, K, M, N, n_sel, max(E_loc, 1))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    w_nb2 = w_local.stride(0) * es if E_loc > 0 else 0
    _check(_L.lib().feml_b200_mul_mat_id_shard(int(wtype), _ptr(w_local), w_local.stride(1) * es, w_nb2, n_experts,
                                               shard, n_shards, _ptr(x), x.stride(0) * 4, _ptr(ids),
                                               ids.stride(0) * 4, n_sel, _ptr(out), out.stride(1) * 4,
                                               out.stride(0) * 4, K, M, N, _ptr(workspace), workspace.numel(), st,
                                               _stream()))
    return out


def _ptr_array(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(v)) for v in ptrs])
    return arr


def mul_mat_peer(wtype, w_local, x, K, dst0_ptrs, dst1_ptrs, flag_ptrs, dst_nb1, counter, epoch, status=None):
    """feml_b200_mul_mat_peer: this rank's rows of a row-sharded decode
    mul_mat stored straight into every rank's output buffer (raw device
    pointers, own memory or IPC mappings), then every rank's flag raised."""
    M, N = w_local.shape[0], x.shape[0]
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    n = len(flag_ptrs)
    _check(_L.lib().feml_b200_mul_mat_peer(int(wtype), _ptr(w_local), w_local.stride(0) * w_local.element_size(),
                                           _ptr(x), x.stride(0) * 4, _ptr_array(dst0_ptrs), _ptr_array(dst1_ptrs),
                                           _ptr_array(flag_ptrs), n, dst_nb1, _ptr(counter), _ptr(epoch), K, M, N, st,
                                           _stream()))


def mul_mat_id_peer(wtype, w_local, x, ids, K, n_experts, shard, n_shards, dst0_ptrs, dst1_ptrs, flag_ptrs,
                    dst_nb1, dst_nb2, M, counter, epoch, workspace, status=None, owner_tokens=0):
    """feml_b200_mul_mat_id_peer(_owned): this shard's experts of an
    expert-sharded mul_mat_id, every output slot stored straight into every
    rank's output buffer of this step (owner_tokens == 0) or only into the
    buffer of the rank that owns its token (token t on rank t // owner_tokens),
    then every rank's flag raised."""
    E_loc = w_local.shape[0]
    if E_loc != local_experts(n_experts, shard, n_shards):
        raise FemlError("msg", f"mul_mat_id_peer: shard {shard}/{n_shards} of {n_experts} experts holds "
                               f"{local_experts(n_experts, shard, n_shards)} experts, got {E_loc}")
    N, n_sel = ids.shape
    es = w_local.element_size()
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    _check(_L.lib().feml_b200_mul_mat_id_peer_owned(int(wtype), _ptr(w_local), w_local.stride(1) * es,
                                                    w_local.stride(0) * es, n_experts, shard, n_shards, _ptr(x),
                                                    x.stride(0) * 4, _ptr(ids), ids.stride(0) * 4, n_sel,
                                                    _ptr_array(dst0_ptrs), _ptr_array(dst1_ptrs),
                                                    _ptr_array(flag_ptrs), len(flag_ptrs), dst_nb1, dst_nb2,
                                                    int(owner_tokens), _ptr(counter), _ptr(epoch), K, M, N,
                                                    _ptr(workspace), workspace.numel(), st, _stream()))


def peer_wait(flag, epoch, n_ranks, status=None, timeout_us=None):
    """Enqueue the end of a fused step: wait for every rank's signal (bounded
    by `timeout_us`, default about a second; on expiry bit 0 of `status` is
    set and the stream continues)."""
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    if timeout_us is None:
        _check(_L.lib().feml_b200_peer_wait(_ptr(flag), _ptr(epoch), n_ranks, st, _stream()))
    else:
        _check(_L.lib().feml_b200_peer_wait_timeout(_ptr(flag), _ptr(epoch), n_ranks, int(timeout_us), st,
                                                    _stream()))


def moe_route(ids, n_experts, status=None):
    """ids int32 [N, n_sel] -> (counts, offsets, rows) int32 device tensors."""
    N, n_sel = ids.shape
    dev = ids.device
    counts = torch.zeros(n_experts, dtype=torch.int32, device=dev)
    offsets = torch.zeros(n_experts, dtype=torch.int32, device=dev)
    rows = torch.full((N * n_sel,), -1, dtype=torch.int32, device=dev)
    st = _ptr(status) if status is not None else ctypes.c_void_p()
    _check(_L.lib().feml_b200_moe_route(_ptr(ids), ids.stride(0) * 4, n_sel, N, n_experts, _ptr(counts),
                                        _ptr(offsets), _ptr(rows), st, _stream()))
    return counts, offsets, rows


def block_dots(wtype, w, xq, K):
    """Per-block int32 sums: w uint8 [M, row_bytes], xq uint8 [N, q8 row bytes]
    -> int32 [M, N, K/32]."""
    M, N = w.shape[0], xq.shape[0]
    out = torch.empty((M, N, K // 32), dtype=torch.int32, device=w.device)
    _check(_L.lib().feml_b200_block_dots(int(wtype), _ptr(w), w.stride(0), _ptr(xq), K, M, N, _ptr(out), _stream()))
    return out


__all__ = ["quantize", "mul_mat", "mul_mat_launches", "mul_mat_workspace", "mul_mat_noalloc", "mul_mat_noalloc_limit", "mul_mat_id", "mul_mat_id_workspace", "mul_mat_id_shard",
           "local_experts", "mul_mat_peer", "mul_mat_id_peer", "peer_wait", "moe_route",
           "block_dots", "row_bytes", "FemlError"]
