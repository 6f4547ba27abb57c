"""Tensor-parallel decode layers over torch.distributed (NCCL on NVLink/NVSwitch).

One process per GPU.  Partitioning (the reference has no multi-GPU code; this
follows the decode layer shapes it benchmarks):

* column-parallel W4A16 (K x N, N sharded): rank r owns output rows
  [r*N/g, (r+1)*N/g) of wq/scales/zeros; x is replicated; each rank computes
  its bf16 y shard and an all-gather rebuilds y [M, N];
* row-parallel W4A16 (K sharded): rank r owns K columns [r*K/g, (r+1)*K/g)
  (a whole number of 128-wide groups) and the matching slice of x; each rank
  computes fp32 partial sums (no bf16 rounding), an fp32 all-reduce adds
  them, and the sum is rounded to bf16 once;
* GQA decode attention, KV heads sharded: rank r owns KV heads
  [r*Hkv/g, (r+1)*Hkv/g) and their query heads; an all-gather over heads
  rebuilds o [B, Hq, D].

The per-rank compute is the sm_100a kernel path (focal_b200.w4a16_linear /
w4a16_linear_f32 / gqa_decode_attention).  ``local_ops`` lets a caller
substitute the per-rank compute; the gloo tests use it to check the sharding
and collectives on CPU.

With a ``TpGroup`` the two W4A16 layers run fused instead: one kernel per
layer computes the shard and exchanges its row blocks with the other ranks
over NVLink peer memory (focal_w4a16_gemv_allgather / _allreduce in
include/focal_b200.h), with no NCCL call on the data path.  The group's
buffers are created and mapped by the library (CUDA IPC handles, exchanged
once with ``all_gather_object``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

GROUP = 128


@dataclass
class LocalOps:
    linear_bf16: callable
    linear_f32: callable
    attention: callable


def cuda_ops() -> LocalOps:
    import focal_b200 as F

    return LocalOps(F.w4a16_linear, F.w4a16_linear_f32, F.gqa_decode_attention)


# -------------------------------------------------------------- partitioning
def column_shard(wq, scales, zeros, rank: int, world: int):
    """Rows [r*N/g, (r+1)*N/g) of an N-sharded (column-parallel) projection."""
    N = wq.shape[0]
    if N % world or (N // world) % 64:
        raise ValueError(f"N={N} does not split into {world} shards of a multiple of 64 rows")
    n = N // world
    sl = slice(rank * n, (rank + 1) * n)
    return wq[sl].contiguous(), scales[sl].contiguous(), zeros[sl].contiguous()


def row_shard(wq, scales, zeros, rank: int, world: int):
    """K columns [r*K/g, (r+1)*K/g) of a K-sharded (row-parallel) projection."""
    K = wq.shape[1] * 8
    if K % world or (K // world) % 256:
        raise ValueError(f"K={K} does not split into {world} shards of a multiple of 256")
    k = K // world
    return (wq[:, rank * k // 8:(rank + 1) * k // 8].contiguous(),
            scales[:, rank * k // GROUP:(rank + 1) * k // GROUP].contiguous(),
            zeros[:, rank * k // GROUP:(rank + 1) * k // GROUP].contiguous())


def x_shard(x, rank: int, world: int):
    k = x.shape[1] // world
    return x[:, rank * k:(rank + 1) * k].contiguous()


def heads_shard(q, k_cache, v_cache, rank: int, world: int):
    Hq, Hkv = q.shape[1], k_cache.shape[1]
    if Hkv % world:
        raise ValueError(f"Hkv={Hkv} does not split into {world} shards")
    hk = Hkv // world
    hq = Hq // world
    return (q[:, rank * hq:(rank + 1) * hq].contiguous(),
            k_cache[:, rank * hk:(rank + 1) * hk].contiguous(),
            v_cache[:, rank * hk:(rank + 1) * hk].contiguous())


# ----------------------------------------------------------------- collectives
def world_size(group=None) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def rank_of(group=None) -> int:
    return dist.get_rank(group) if dist.is_initialized() else 0


def gather_columns(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """[M, N/g] shards -> [M, N] in rank order (one all_gather_into_tensor)."""
    world = world_size(group)
    if world == 1:
        return y_local
    M, n = y_local.shape
    out = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(out, y_local.contiguous(), group=group)
    return out.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)


def gather_heads(o_local: torch.Tensor, group=None) -> torch.Tensor:
    """[B, Hq/g, D] shards -> [B, Hq, D] in rank order."""
    world = world_size(group)
    if world == 1:
        return o_local
    B, h, D = o_local.shape
    out = torch.empty((world * B, h, D), dtype=o_local.dtype, device=o_local.device)
    dist.all_gather_into_tensor(out, o_local.contiguous(), group=group)
    return out.view(world, B, h, D).permute(1, 0, 2, 3).reshape(B, world * h, D)


def reduce_partials(partial_f32: torch.Tensor, group=None) -> torch.Tensor:
    """Sum fp32 partials over ranks, then round once to bf16."""
    if world_size(group) > 1:
        dist.all_reduce(partial_f32, op=dist.ReduceOp.SUM, group=group)
    return partial_f32.to(torch.bfloat16)


# ------------------------------------------------------- fused peer-memory group
class _DeviceBytes:
    """A raw device buffer seen as a torch uint8 tensor (zero-copy, through the
    CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class TpGroup:
    """Peer-memory buffers of a tensor-parallel group for the fused linears.

    Each rank creates one zero-filled buffer of
    ``focal_tp_buffer_size(world, max_m, max_n)`` bytes on its GPU
    (focal_tp_buffer_create), sends its CUDA IPC handle to the other ranks
    (``all_gather_object``), and maps theirs for its own GPU
    (focal_tp_buffer_open).  Every rank must make the same sequence of fused
    calls with the same shapes, on one stream per rank (the buffers hold
    per-call state), and each rank needs its own GPU.  ``world == 1`` (no
    process group) runs the same kernels against the local buffer alone.
    """

    def __init__(self, max_m: int = 8, max_n: int = 65536, group=None, device=None):
        import ctypes

        from . import _lib

        self.group = group
        self.world = world_size(group)
        self.rank = rank_of(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        L = _lib.lib()
        self.bytes = int(L.focal_tp_buffer_size(self.world, max_m, max_n))
        if self.bytes == 0:
            raise ValueError(f"no tensor-parallel buffer for world={self.world} M<={max_m} N<={max_n}")
        if self.world > 1:
            # ranks whose kernels wait on one another must not share a GPU
            uuids = [None] * self.world
            dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
            if len(set(uuids)) != self.world:
                raise ValueError(f"tensor-parallel ranks share a GPU ({uuids}); every rank needs its own")
        handle = (ctypes.c_uint8 * 64)()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("focal_tp_buffer_create", self.bytes, ctypes.byref(ptr), handle)
            self._own = ptr.value
            self._opened = []
            peers = [0] * self.world
            peers[self.rank] = self._own
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
                for q in range(self.world):
                    if q != self.rank:
                        p = ctypes.c_void_p()
                        _lib.call("focal_tp_buffer_open", (ctypes.c_uint8 * 64).from_buffer_copy(handles[q]),
                                  ctypes.byref(p))
                        peers[q] = p.value
                        self._opened.append(p.value)
                dist.barrier(group=group)  # every buffer is zero and mapped before any rank stores into it
        # this rank's buffer as a tensor: [0:4] completed calls, [4:8] CTAs done
        self.buf = torch.as_tensor(_DeviceBytes(self._own, self.bytes), device=self.device)
        self.comm = _lib.TpComm()
        for q, p in enumerate(peers):
            self.comm.peer[q] = p
        self.comm.bytes = self.bytes
        self.comm.world = self.world
        self.comm.rank = self.rank
        self._ws = None
        self._ws_bytes = 0

    def _workspace(self, M, K, N):
        from . import _lib

        need = int(_lib.lib().focal_w4a16_workspace_size(M, K, N))
        if need > self._ws_bytes:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
            self._ws_bytes = need
        return self._ws

    def _call(self, name, x, wq, scales, zeros, y):
        import ctypes

        from . import _lib

        M, K = x.shape
        N = wq.shape[0]
        ws = self._workspace(M, K, N)
        _lib.call(name, x.data_ptr(), wq.data_ptr(), scales.data_ptr(), zeros.data_ptr(), y.data_ptr(), M, K, N,
                  ctypes.byref(self.comm), ws.data_ptr(), self._ws_bytes,
                  torch.cuda.current_stream(self.device).cuda_stream)
        return y

    def allgather_linear(self, x, wq, scales, zeros) -> torch.Tensor:
        """Column-parallel shard + all-gather in one kernel: y [M, world*N] bf16."""
        M, N = x.shape[0], wq.shape[0]
        y = torch.empty((M, self.world * N), dtype=torch.bfloat16, device=x.device)
        return self._call("focal_w4a16_gemv_allgather", x, wq, scales, zeros, y)

    def allreduce_linear(self, x_local, wq, scales, zeros) -> torch.Tensor:
        """Row-parallel shard + fp32 all-reduce in one kernel: y [M, N] bf16."""
        M, N = x_local.shape[0], wq.shape[0]
        y = torch.empty((M, N), dtype=torch.bfloat16, device=x_local.device)
        return self._call("focal_w4a16_gemv_allreduce", x_local, wq, scales, zeros, y)

    def close(self):
        """Unmap the peers' buffers and free this rank's, once every rank is
        done with the group (collective over the group's ranks)."""
        from . import _lib

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank stores into a buffer after this
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("focal_tp_buffer_close", p)
            self._opened = []
            if self.world > 1:
                dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
            self.buf = None
            _lib.call("focal_tp_buffer_destroy", self._own)
        self._own = None


# ---------------------------------------------------------------------- layers
class ColumnParallelW4A16:
    """y = x W^T with W sharded over N; returns the full bf16 y on every rank."""

    def __init__(self, wq, scales, zeros, group=None, ops: LocalOps | None = None, gather=True,
                 fused: TpGroup | None = None):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_size(group)
        self.shard = column_shard(wq, scales, zeros, self.rank, self.world)
        self.ops = ops or cuda_ops()
        self.gather = gather
        self.fused = fused

    def local(self, x):
        return self.ops.linear_bf16(x, *self.shard)

    def __call__(self, x):
        if self.fused is not None and self.gather:
            return self.fused.allgather_linear(x, *self.shard)
        y = self.local(x)
        return gather_columns(y, self.group) if self.gather else y


class RowParallelW4A16:
    """y = x W^T with W (and x) sharded over K; fp32 all-reduce, one bf16 rounding."""

    def __init__(self, wq, scales, zeros, group=None, ops: LocalOps | None = None,
                 fused: TpGroup | None = None):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_size(group)
        self.shard = row_shard(wq, scales, zeros, self.rank, self.world)
        self.ops = ops or cuda_ops()
        self.fused = fused

    def local(self, x_local):
        return self.ops.linear_f32(x_local, *self.shard)

    def __call__(self, x_local):
        if self.fused is not None:
            return self.fused.allreduce_linear(x_local, *self.shard)
        return reduce_partials(self.local(x_local), self.group)


class HeadParallelAttention:
    """GQA decode attention with KV heads sharded; returns the full o."""

    def __init__(self, group=None, ops: LocalOps | None = None):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_size(group)
        self.ops = ops or cuda_ops()

    def __call__(self, q_local, k_local, v_local, scale=None):
        return gather_heads(self.ops.attention(q_local, k_local, v_local, scale), self.group)
