"""One rank of the multi-GPU check of the fused tensor-parallel linears; run by
tests/test_gpu_tp_fused.py as ``torchrun --nproc-per-node G`` (one process per
GPU, NCCL only for the checks themselves).

Per rank and case, repeated twice so both receive halves are used:
* column-parallel: the fused all-gather equals the NCCL all-gather of the
  plain bf16 shards, bit for bit;
* row-parallel: the fused all-reduce equals bf16 of the rank-order fp32 sum
  of the plain fp32 partials, bit for bit;
* every rank holds the same bits; the small cases also match the oracle of
  the unsharded layer within the linear's tolerance (atol 2e-2, rtol 1e-2).
"""
import ctypes
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from focal_b200 import _lib  # noqa: E402
from focal_b200.tp import TpGroup  # noqa: E402
from oracle import w4a16 as ow  # noqa: E402
from tests import _capi as C  # noqa: E402

ATOL, RTOL = 2e-2, 1e-2

# (kind, M, K, N) of the unsharded layer; "col" shards N, "row" shards K
CASES = [("col", 8, 4096, 8192), ("row", 8, 8192, 4096), ("col", 2, 1024, 512), ("row", 3, 2048, 512),
         ("col", 8, 8192, 28672), ("row", 8, 28672, 8192), ("col", 1, 11008, 4096), ("row", 5, 4096, 11008)]
ORACLE_MAX_MACS = 8 * 8192 * 8192


def gather(t):
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t.contiguous())
    return out


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    group = TpGroup(max_m=8, max_n=16384, device=dev)
    for rep in range(2):
        for i, (kind, M, K, N) in enumerate(CASES):
            x, wq, s, z = ow.baseline_case(M, K, N, seed=700 + i)
            if kind == "col":
                n = N // world
                rows = slice(rank * n, (rank + 1) * n)
                xs, ws, ss, zs = x, wq[rows], s[rows], z[rows]
            else:
                k = K // world
                xs = x[:, rank * k:(rank + 1) * k]
                ws, ss, zs = wq[:, rank * k // 8:(rank + 1) * k // 8], s[:, rank * k // 128:(rank + 1) * k // 128], \
                    z[:, rank * k // 128:(rank + 1) * k // 128]
            dx = C.to_dev_bf16(xs, dev)
            dw, ds, dz = (C.to_dev(a, dev) for a in (ws, ss, zs))
            if kind == "col":
                y = group.allgather_linear(dx, dw, ds, dz)
                want = torch.cat(gather(C.gemv(dx, dw, ds, dz)), dim=1)
            else:
                y = group.allreduce_linear(dx, dw, ds, dz)
                parts = gather(C.gemv(dx, dw, ds, dz, out_dtype=torch.float32))
                acc = parts[0].clone()
                for p in parts[1:]:
                    acc += p
                want = acc.to(torch.bfloat16)
            assert torch.equal(y.view(torch.int16), want.view(torch.int16)), (rank, rep, kind, M, K, N)
            for other in gather(y):
                assert torch.equal(other.view(torch.int16), y.view(torch.int16)), (rank, rep, kind, M, K, N)
            if rep == 0 and M * K * N <= ORACLE_MAX_MACS:
                rep_ = ow.allclose_report(C.bf16_bits(y), ow.linear(x, wq, s, z), ATOL, RTOL)
                assert rep_["allclose"], (rank, kind, M, K, N, rep_)
    torch.cuda.synchronize(dev)
    status = ctypes.c_int(-1)
    assert _lib.lib().focal_device_status(status) == 0 and status.value == 0, status.value
    state = group.buf[:8].view(torch.int32).cpu().tolist()
    assert state == [2 * len(CASES), 0], state
    group.close()
    print(f"tp fused ok rank {rank} world {world}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
