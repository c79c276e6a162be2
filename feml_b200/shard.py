"""Multi-GPU mul_mat / mul_mat_id: one process per GPU over torch.distributed.

The reference runs one backend per process and has no multi-device code
(feml-core/src/backend.rs:96-165 is a single-device trait), so these wrappers
are new. They shard the two operators of the path the natural way:

* `RowShardedMulMat` -- rank r owns the weight rows [r*R, min(M, (r+1)*R)),
  R = ceil(M / world). In the ggml layout those rows are one contiguous byte
  range (feml-core/src/layout.rs:38-40). Each rank computes its [N, R] slice
  of y = W x straight into its all-gather send buffer, one all-gather over
  NCCL assembles [world, N, R], and a permute gives y [N, M] on every rank.
  With N == 1 the gathered buffer already is y (no permute).
  With `fused=True` and a decode shape (N <= 8, N*K <= 16384) the all-gather
  is fused into the kernel instead: every rank stores its rows straight into
  every rank's output buffer over NVLink (peer pointers from CUDA IPC, mapped
  once into this device's context with peer access), raises each rank's flag, and a
  one-thread wait kernel ends the step when all ranks have signalled
  (feml_b200_mul_mat_peer / feml_b200_peer_wait; bounded waits; no NCCL on
  the data path). Outputs alternate between two buffers by step.
* `ExpertShardedMulMatId` -- rank r owns the experts e with e % world == r
  (local index e // world). Each rank computes the dst slots routed to its
  experts (feml_b200_mul_mat_id_shard leaves the other slots untouched in a
  zeroed buffer) and the combine brings every slot to where it is needed.
  Every slot has exactly one non-zero contributor, so the combine is exact;
  invalid expert ids give zero slots, as on one device. Two combines:
    - combine="replicate": every rank ends with all N tokens' slots (a sum
      all-reduce; fused: the GEMM epilogue stores every slot into every
      rank's buffer over NVLink, feml_b200_mul_mat_id_peer);
    - combine="owner": token t belongs to rank t // T, T = ceil(max_tokens /
      world), and each rank ends with only its own tokens' slots (the
      all-to-all of expert parallelism; collective form: a sum all-reduce
      sliced to the rank's tokens; fused: the epilogue stores each slot only
      into its owner's buffer, feml_b200_mul_mat_id_peer_owned, so a rank
      sends about 1/world of the slot tensor instead of all of it to every
      peer).
  `fused=True` needs quantized weights, K % 256 == 0, at most `max_tokens`
  tokens and `max_selected` experts per token; the flag / epoch wait of the
  row-sharded path ends the step.

The compute step defaults to the CUDA entry points of libfeml_b200.so
(feml_b200.ops); `compute` / `compute_id` can be replaced, which the CPU
tests use to run the sharding and collective logic on gloo ranks.
"""
import torch
import torch.distributed as dist

from . import DType, FemlError


def row_range(M, rank, world):
    """Rows [lo, hi) of an M-row weight owned by `rank`, and the padded
    per-rank row count R = ceil(M / world) every rank gathers."""
    R = -(-M // world)
    lo = min(M, rank * R)
    return lo, min(M, lo + R), R


def local_experts(n_experts, shard, n_shards):
    """Experts owned by `shard`: e = shard, shard + n_shards, ..."""
    return max(0, (n_experts - shard + n_shards - 1) // n_shards)


def _cuda_mul_mat(wtype, w_local, x, K, out):
    from . import ops
    return ops.mul_mat(wtype, w_local, x, K, out=out)


def _cuda_mul_mat_id(wtype, w_local, x, ids, K, n_experts, shard, n_shards, out):
    from . import ops
    return ops.mul_mat_id_shard(wtype, w_local, x, ids, K, n_experts, shard, n_shards, out)


def _world(group):
    return dist.get_rank(group), dist.get_world_size(group)


def _gather(out, send, group):
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, send, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), send, group=group)


class _PeerBuffers:
    """The peer-memory state of a fused step: two output buffers, a step flag,
    a grid counter and an epoch per rank. Every rank maps every other rank's
    buffers and flag into its own device's context with peer access (CUDA IPC
    handles of the torch allocations, exchanged with all_gather_object and
    opened through feml_b200_ipc_open). dst0 / dst1 / flags hold, per rank,
    the address this rank's kernels write (byte `offset` into the buffers)."""

    def __init__(self, shape, device, group, offset=0):
        import ctypes
        from . import _check, _lib
        self.rank, world = _world(group)
        self.bufs = [torch.zeros(shape, dtype=torch.float32, device=device) for _ in range(2)]
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.steps = 0
        torch.cuda.synchronize(device)
        mine = []
        for t in (self.bufs[0], self.bufs[1], self.flag):
            handle = ctypes.create_string_buffer(64)
            off = ctypes.c_uint64()
            _check(_lib.lib().feml_b200_ipc_export(ctypes.c_void_p(t.data_ptr()), handle, 64, ctypes.byref(off)))
            mine.append((handle.raw, off.value))
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        opened = {}  # one mapping per peer allocation
        ptrs = []
        for r, shared in enumerate(everyone):
            if r == self.rank:
                ptrs.append([self.bufs[0].data_ptr(), self.bufs[1].data_ptr(), self.flag.data_ptr()])
                continue
            row = []
            for handle, off in shared:
                if handle not in opened:
                    base = ctypes.c_void_p()
                    _check(_lib.lib().feml_b200_ipc_open(handle, len(handle), ctypes.byref(base)))
                    opened[handle] = base.value
                row.append(opened[handle] + off)
            ptrs.append(row)
        self.opened = list(opened.values())
        self.dst0 = [p[0] + offset for p in ptrs]
        self.dst1 = [p[1] + offset for p in ptrs]
        self.flags = [p[2] for p in ptrs]
        dist.barrier(group=group)

    def finish(self, world):
        """Enqueue the wait for every rank's signal; returns this step's buffer."""
        from . import ops
        ops.peer_wait(self.flag, self.epoch, world)
        self.steps += 1
        return self.bufs[self.steps & 1]

    def close(self):
        from . import _lib
        torch.cuda.synchronize()
        for base in self.opened:
            _lib.lib().feml_b200_ipc_close(base)
        self.opened = []


class RowShardedMulMat:
    """y [N, M] = W x with W row-sharded across the ranks of `group`.

    `w` is either the full weight (uint8 [M, row_bytes], or f32 [M, K] for
    F32) from which this rank keeps its rows, or (local=True) this rank's
    rows already.
    """

    def __init__(self, wtype, w, K, M, group=None, local=False, compute=None, fused=False, max_tokens=4):
        self.wtype = DType(wtype)
        self.K, self.M = K, M
        self.group = group
        self.rank, self.world = _world(group)
        self.lo, self.hi, self.R = row_range(M, self.rank, self.world)
        self.fused = fused
        self.max_tokens = max_tokens
        self._peer = None
        if local:
            if w.shape[0] != self.hi - self.lo:
                raise FemlError("shape", f"rank {self.rank} holds rows [{self.lo}, {self.hi}), "
                                         f"got {w.shape[0]} rows")
            self.w_local = w
        else:
            if w.shape[0] != M:
                raise FemlError("shape", f"weight has {w.shape[0]} rows, expected {M}")
            self.w_local = w[self.lo:self.hi]
        self.compute = compute or _cuda_mul_mat

    def _setup_peers(self, device):
        if self.hi <= self.lo:
            raise FemlError("shape", f"fused row sharding needs rows on every rank (rank {self.rank} has none)")
        self._peer = _PeerBuffers((self.max_tokens, self.M), device, self.group, 4 * self.lo)

    def close(self):
        """Unmap the peers' buffers (after the last fused step has finished)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def _fused_ok(self, N):
        return (self.fused and N <= self.max_tokens and N * self.K <= 16384 and self.wtype != DType.F32
                and self.compute is _cuda_mul_mat)

    def __call__(self, x):
        N = x.shape[0]
        if x.shape[1] != self.K:
            raise FemlError("shape", f"activation has K={x.shape[1]}, expected {self.K}")
        if self._fused_ok(N):
            from . import ops
            if self._peer is None:
                self._setup_peers(x.device)
            pe = self._peer
            ops.mul_mat_peer(self.wtype, self.w_local, x, self.K, pe.dst0, pe.dst1, pe.flags, 4 * self.M,
                             pe.counter, pe.epoch)
            return pe.finish(self.world)[:N]
        send = torch.empty((N, self.R), dtype=torch.float32, device=x.device)
        m_loc = self.hi - self.lo
        if m_loc < self.R:
            send[:, m_loc:].zero_()
        if m_loc:
            self.compute(self.wtype, self.w_local, x, self.K, send[:, :m_loc])
        gathered = torch.empty((self.world, N, self.R), dtype=torch.float32, device=x.device)
        _gather(gathered, send, self.group)
        if N == 1:
            return gathered.view(1, self.world * self.R)[:, :self.M]
        return gathered.permute(1, 0, 2).reshape(N, self.world * self.R)[:, :self.M]


class ExpertShardedMulMatId:
    """out = mul_mat_id(W, x, ids) with experts sharded across the ranks of
    `group` (expert e on rank e % world): [N, n_sel, M] on every rank
    (combine="replicate"), or this rank's tokens [hi - lo, n_sel, M] with
    (lo, hi) = token_range(N) (combine="owner").

    `w` is either all experts (uint8 [E, M, row_bytes]) from which this rank
    keeps its own, or (local=True) this rank's experts already, in local
    order.
    """

    def __init__(self, wtype, w, K, n_experts, group=None, local=False, compute_id=None, fused=False,
                 max_tokens=512, max_selected=8, combine="replicate"):
        if combine not in ("replicate", "owner"):
            raise FemlError("msg", f"combine must be 'replicate' or 'owner', got {combine!r}")
        self.wtype = DType(wtype)
        self.K, self.E = K, n_experts
        self.group = group
        self.rank, self.world = _world(group)
        self.fused = fused
        self.combine = combine
        self.max_tokens, self.max_selected = max_tokens, max_selected
        self.owner_tokens = -(-max_tokens // self.world)
        self._peer = None
        n_loc = local_experts(n_experts, self.rank, self.world)
        if local:
            if w.shape[0] != n_loc:
                raise FemlError("shape", f"rank {self.rank} owns {n_loc} experts, got {w.shape[0]}")
            self.w_local = w
        else:
            if w.shape[0] != n_experts:
                raise FemlError("shape", f"weight has {w.shape[0]} experts, expected {n_experts}")
            self.w_local = w[self.rank::self.world]
        self.M = w.shape[1]
        self.compute_id = compute_id or _cuda_mul_mat_id

    def token_range(self, N):
        """Tokens [lo, hi) whose slots this rank holds after an owner combine."""
        if N > self.max_tokens:
            raise FemlError("shape", f"{N} tokens exceed max_tokens={self.max_tokens}")
        lo = min(N, self.rank * self.owner_tokens)
        return lo, min(N, lo + self.owner_tokens)

    def close(self):
        """Unmap the peers' buffers (after the last fused step has finished)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def _fused_ok(self, N, n_sel):
        return (self.fused and N <= self.max_tokens and n_sel <= self.max_selected and self.K % 256 == 0
                and self.wtype != DType.F32 and self.compute_id is _cuda_mul_mat_id and self.world <= 8)

    def __call__(self, x, ids):
        N, n_sel = ids.shape
        if x.shape[0] != N or x.shape[1] != self.K:
            raise FemlError("shape", f"activation {tuple(x.shape)} does not match ids {tuple(ids.shape)} / K={self.K}")
        owner = self.combine == "owner"
        lo, hi = self.token_range(N) if owner else (0, N)
        if self._fused_ok(N, n_sel):
            from . import ops
            if self._peer is None:
                if self.w_local.shape[0] < 1:
                    raise FemlError("shape", f"fused expert sharding needs an expert on every rank "
                                             f"(rank {self.rank} has none)")
                rows = self.owner_tokens if owner else self.max_tokens
                self._peer = _PeerBuffers((rows, self.max_selected, self.M), x.device, self.group)
                self._ws = torch.empty(ops.mul_mat_id_workspace(self.wtype, self.K, self.M, self.max_tokens,
                                                                self.max_selected, self.w_local.shape[0]),
                                       dtype=torch.uint8, device=x.device)
            pe = self._peer
            # slot (t, s) at t * nb2 + s * nb1 of a [tokens, n_sel, M] view of each buffer
            nb1, nb2 = 4 * self.M, 4 * self.M * n_sel
            ops.mul_mat_id_peer(self.wtype, self.w_local, x, ids, self.K, self.E, self.rank, self.world, pe.dst0,
                                pe.dst1, pe.flags, nb1, nb2, self.M, pe.counter, pe.epoch, self._ws,
                                owner_tokens=self.owner_tokens if owner else 0)
            buf = pe.finish(self.world)
            n_out = hi - lo
            return buf.view(-1)[:n_out * n_sel * self.M].view(n_out, n_sel, self.M)
        out = torch.zeros((N, n_sel, self.M), dtype=torch.float32, device=x.device)
        self.compute_id(self.wtype, self.w_local, x, ids, self.K, self.E, self.rank, self.world, out)
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out[lo:hi] if owner else out


__all__ = ["RowShardedMulMat", "ExpertShardedMulMatId", "row_range", "local_experts"]
