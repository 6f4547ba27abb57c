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


# ---------------------------------------------------------------------- layers
class ColumnParallelW4A16:
    """y = x W^T with W sharded over N; returns the full bf16 y on every rank."""

    def __init__(self, wq, scales, zeros, group=None, ops: LocalOps | None = None, gather=True):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_size(group)
        self.shard = column_shard(wq, scales, zeros, self.rank, self.world)
        self.ops = ops or cuda_ops()
        self.gather = gather

    def local(self, x):
        return self.ops.linear_bf16(x, *self.shard)

    def __call__(self, x):
        y = self.local(x)
        return gather_columns(y, self.group) if self.gather else y


class RowParallelW4A16:
    """y = x W^T with W (and x) sharded over K; fp32 all-reduce, one bf16 rounding."""

    def __init__(self, wq, scales, zeros, group=None, ops: LocalOps | None = None):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_size(group)
        self.shard = row_shard(wq, scales, zeros, self.rank, self.world)
        self.ops = ops or cuda_ops()

    def local(self, x_local):
        return self.ops.linear_f32(x_local, *self.shard)

    def __call__(self, x_local):
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
