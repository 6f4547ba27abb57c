"""The fused tensor-parallel linears (focal_w4a16_gemv_allgather / _allreduce),
called through the C ABI.

One GPU: a group of one rank runs the same kernels (stores into its own
buffer, releases and waits on its own flags); the outputs must equal the plain
linear's bit for bit, over repeated calls that alternate the two receive
halves and change shape.  Two or more GPUs: tests/tp_fused_worker.py under
torchrun checks, on every rank, that the fused all-gather equals the NCCL
all-gather of the plain shards and that the fused all-reduce equals the rank-
order fp32 sum of the plain fp32 partials, both bit for bit, and both against
the oracle within the linear's tolerance.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w4a16 as ow
from tests import _capi as C

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_single_rank_group_matches_plain_linear(cuda):
    from focal_b200 import _lib
    from focal_b200.tp import TpGroup

    group = TpGroup(max_m=8, max_n=8192, device=cuda)
    cases = [(8, 4096, 8192), (1, 8192, 4096), (4, 4096, 4096), (8, 11008, 4096), (2, 1024, 192)]
    for it in range(3):
        for i, (M, K, N) in enumerate(cases):
            x, wq, s, z = (C.to_dev_bf16(a, cuda) if j == 0 else C.to_dev(a, cuda)
                           for j, a in enumerate(ow.baseline_case(M, K, N, seed=300 + 10 * i + it)))
            plain = C.gemv(x, wq, s, z)
            ag = group.allgather_linear(x, wq, s, z)
            ar = group.allreduce_linear(x, wq, s, z)
            assert torch.equal(ag.view(torch.int16), plain.view(torch.int16)), (M, K, N, it)
            assert torch.equal(ar.view(torch.int16), plain.view(torch.int16)), (M, K, N, it)
    torch.cuda.synchronize()
    status = __import__("ctypes").c_int(-1)
    assert _lib.lib().focal_device_status(status) == 0 and status.value == 0
    # two kernels per case and iteration advanced the group's epoch
    state = group.buf[:8].view(torch.int32).cpu().tolist()
    assert state == [2 * 3 * len(cases), 0]
    group.close()


def test_group_rejects_bad_arguments(cuda):
    import ctypes

    from focal_b200 import _lib
    from focal_b200.tp import TpGroup

    group = TpGroup(max_m=8, max_n=512, device=cuda)
    x, wq, s, z = (C.to_dev_bf16(a, cuda) if j == 0 else C.to_dev(a, cuda)
                   for j, a in enumerate(ow.baseline_case(8, 1024, 1024, seed=1)))
    y = torch.empty((8, 1024), dtype=torch.bfloat16, device=cuda)
    ws, n = C.w4a16_workspace(8, 1024, 1024, cuda)
    L = _lib.lib()
    rc = L.focal_w4a16_gemv_allreduce(x.data_ptr(), wq.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                      8, 1024, 1024, ctypes.byref(group.comm), ws.data_ptr(), n, C.stream_ptr())
    assert rc == _lib.FOCAL_ERR_WORKSPACE and "tensor-parallel buffers too small" in _lib.last_error()
    bad = _lib.TpComm()
    bad.world, bad.rank, bad.bytes = 2, 2, group.bytes
    rc = L.focal_w4a16_gemv_allgather(x.data_ptr(), wq.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                      8, 1024, 512, ctypes.byref(bad), ws.data_ptr(), n, C.stream_ptr())
    assert rc == _lib.FOCAL_ERR_INVALID_VALUE and "out of range" in _lib.last_error()
    group.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_group_over_nvlink():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
           str(ROOT / "tests" / "tp_fused_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    errors = [ln for ln in r.stderr.splitlines() if "rror" in ln or "rank" in ln][:40]
    assert r.returncode == 0, r.stdout[-3000:] + "\n".join(errors)
    assert r.stdout.count("tp fused ok") == 2, r.stdout[-4000:]


@pytest.mark.parametrize("M,K,N", [(1, 1024, 256), (1, 256, 262144)])
def test_missing_peer_times_out_with_status(cuda, M, K, N):
    """A two-rank group whose second buffer nobody ever writes (one GPU, one
    kernel, a word that nothing sets): the bounded poll gives up after about a
    second, the call's device status reads 2 (peer timeout), and the context
    stays usable for later calls.  In the second shape every sub-pipeline
    finishes about seven row blocks; once one poll of a CTA has given up its
    later polls stop at once, so the call still takes about a second, not
    seven."""
    import ctypes
    import time

    from focal_b200 import _lib

    L = _lib.lib()
    nbytes = int(L.focal_tp_buffer_size(2, M, N))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
    comm = _lib.TpComm()
    comm.peer[0], comm.peer[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
    comm.bytes, comm.world, comm.rank = nbytes, 2, 0
    x, wq, s, z = (C.to_dev_bf16(a, cuda) if j == 0 else C.to_dev(a, cuda)
                   for j, a in enumerate(ow.baseline_case(M, K, N, seed=5)))
    y = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ws, n = C.w4a16_workspace(M, K, N, cuda)
    assert L.focal_reset_device_status() == 0
    t0 = time.perf_counter()
    rc = L.focal_w4a16_gemv_allreduce(x.data_ptr(), wq.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                      M, K, N, ctypes.byref(comm), ws.data_ptr(), n, C.stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = ctypes.c_int(-1)
    assert L.focal_device_status(status) == 0 and status.value == 2, status.value
    assert 0.3 < waited < 4, waited
    assert L.focal_reset_device_status() == 0
    # the context still works: a plain call matches the oracle
    assert_close = ow.allclose_report(C.bf16_bits(C.gemv(x, wq, s, z)), ow.linear(*ow.baseline_case(M, K, N, seed=5)),
                                      2e-2, 1e-2)
    assert assert_close["allclose"], assert_close
    assert L.focal_device_status(status) == 0 and status.value == 0


def test_device_failure_is_reported_to_torch_callers(cuda):
    """After a kernel gives up a bounded wait (a two-rank group whose peer never
    writes, as above), the next PyTorch-level call raises instead of returning
    numbers computed on possibly stale counters; it clears the status and
    re-zeroes the cached workspaces, and the call after it matches the oracle."""
    import ctypes

    import focal_w4a16
    from focal_b200 import _lib

    L = _lib.lib()
    M, K, N = 1, 1024, 256
    nbytes = int(L.focal_tp_buffer_size(2, M, N))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
    comm = _lib.TpComm()
    comm.peer[0], comm.peer[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
    comm.bytes, comm.world, comm.rank = nbytes, 2, 0
    case = ow.baseline_case(M, K, N, seed=6)
    x, wq, s, z = (C.to_dev_bf16(a, cuda) if j == 0 else C.to_dev(a, cuda) for j, a in enumerate(case))
    y = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ws, n = C.w4a16_workspace(M, K, N, cuda)
    assert L.focal_reset_device_status() == 0
    focal_w4a16.w4a16_linear(x, wq, s, z)  # the cached workspace exists before the failure
    assert L.focal_w4a16_gemv_allreduce(x.data_ptr(), wq.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                        M, K, N, ctypes.byref(comm), ws.data_ptr(), n, C.stream_ptr()) == 0
    torch.cuda.synchronize()
    peek = ctypes.c_int(-1)
    assert L.focal_device_status_peek(peek) == 0 and peek.value == 2
    with pytest.raises(RuntimeError, match="gave up a bounded device-side wait"):
        focal_w4a16.w4a16_linear(x, wq, s, z)
    assert L.focal_device_status_peek(peek) == 0 and peek.value == 0
    got = focal_w4a16.w4a16_linear(x, wq, s, z)
    rep = ow.allclose_report(C.bf16_bits(got), ow.linear(*case), 2e-2, 1e-2)
    assert rep["allclose"], rep
