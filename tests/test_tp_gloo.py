"""Multi-rank host logic of focal_b200.tp on CPU: world_size-2 gloo ranks.

The per-rank compute is replaced by the CPU oracle (LocalOps injection), so
these tests check the partitioning, the collectives and the reassembly order:
sharded results must equal the unsharded oracle result on every rank.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_ops():
    from focal_b200.tp import LocalOps
    from oracle import attention as oa
    from oracle import w4a16 as ow

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def from_bits(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)

    def lin_bf16(x, wq, s, z):
        return from_bits(ow.linear(bits(x), wq.numpy(), s.numpy(), z.numpy()))

    def lin_f32(x, wq, s, z):
        return torch.from_numpy(ow.linear(bits(x), wq.numpy(), s.numpy(), z.numpy(), out="f32"))

    def attn(q, k, v, scale=None):
        return from_bits(oa.decode_attention(bits(q), bits(k), bits(v), scale))

    return LocalOps(lin_bf16, lin_f32, attn)


def _worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import datetime

        from focal_b200 import tp
        from oracle import attention as oa
        from oracle import w4a16 as ow

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        ops = _oracle_ops()
        to_bf16 = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)  # noqa: E731

        # column-parallel: K=512, N=256 -> 128 rows per rank
        x, wq, s, z = ow.baseline_case(8, 512, 256, seed=1)
        col = tp.ColumnParallelW4A16(torch.from_numpy(wq), torch.from_numpy(s), torch.from_numpy(z), ops=ops)
        y = col(to_bf16(x))
        ref = to_bf16(ow.linear(x, wq, s, z))
        # each rank's shard is an independent sgemm: equal up to fp32 summation order
        assert torch.allclose(y.float(), ref.float(), atol=2e-2, rtol=1e-2), "column"
        assert (y.float() - ref.float()).abs().max() <= ref.float().abs().max() * 2**-7, "column ulp"

        # row-parallel: K=1024 -> 512 per rank; fp32 partials summed, one rounding
        x, wq, s, z = ow.baseline_case(4, 1024, 128, seed=2)
        row = tp.RowParallelW4A16(torch.from_numpy(wq), torch.from_numpy(s), torch.from_numpy(z), ops=ops)
        y = row(tp.x_shard(to_bf16(x), rank, world)).float().numpy().astype(np.float64)
        exact = ow.linear_f64(x, wq, s, z)
        assert np.allclose(y, exact, atol=2e-2, rtol=1e-2), "row"

        # attention, KV heads sharded
        qq, kk, vv = oa.random_case(2, 32, 8, 70, 128, seed=3)
        ql, kl, vl = tp.heads_shard(to_bf16(qq), to_bf16(kk), to_bf16(vv), rank, world)
        o = tp.HeadParallelAttention(ops=ops)(ql, kl, vl)
        ref = to_bf16(oa.decode_attention(qq, kk, vv))
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), "heads"

        # a shard that is not a multiple of the kernel tiles is refused on the host
        try:
            tp.column_shard(torch.from_numpy(wq), torch.from_numpy(s), torch.from_numpy(z), rank, 3)
            raise AssertionError("expected ValueError")
        except ValueError:
            pass
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_tensor_parallel_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_partition_math():
    from focal_b200 import tp

    wq = torch.zeros((28672, 8192 // 8), dtype=torch.int32)
    s = torch.zeros((28672, 64), dtype=torch.float16)
    for g in (1, 2, 4, 8):
        a, b, c = tp.column_shard(wq, s, s, g - 1, g)
        assert a.shape == (28672 // g, 1024) and b.shape == (28672 // g, 64)
    wq = torch.zeros((8192, 28672 // 8), dtype=torch.int32)
    s = torch.zeros((8192, 224), dtype=torch.float16)
    for g in (1, 2, 4, 8):
        a, b, c = tp.row_shard(wq, s, s, 0, g)
        assert a.shape == (8192, 28672 // g // 8) and b.shape == (8192, 224 // g)
    with pytest.raises(ValueError):
        tp.row_shard(wq, s, s, 0, 5)
