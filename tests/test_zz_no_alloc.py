"""focal_w4a16_gemv_noalloc: the linear layer with its fixed per-device scratch
instead of a caller workspace, called through the C ABI.

For callers that cannot allocate device memory where they call the layer.
Collected last (file name) and independent of what ran before: the scratch's
words start at zero when the library loads and every call leaves them at
zero.  Each case makes two calls in a row on different inputs and compares each
with focal_w4a16_gemv (caller workspace) and the oracle.
"""
import numpy as np
import pytest
import torch

from focal_b200 import _lib
from oracle import w4a16 as ow
from tests import _capi as C

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def noalloc(x, wq, scales, zeros):
    M, K = x.shape
    N = wq.shape[0]
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _lib.call("focal_w4a16_gemv_noalloc", C.ptr(x), C.ptr(wq), C.ptr(scales), C.ptr(zeros), C.ptr(y),
              M, K, N, C.stream_ptr())
    return y


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (8, 8192, 11008), (4, 11008, 4096), (2, 8192, 8192)])
def test_noalloc_matches_workspace_entry_point(cuda, M, K, N):
    outs = []
    for call in range(2):
        x, wq, s, z = ow.baseline_case(M, K, N, seed=4000 + 10 * M + call)
        dx, dwq, ds, dz = C.to_dev_bf16(x, cuda), C.to_dev(wq, cuda), C.to_dev(s, cuda), C.to_dev(z, cuda)
        y_na = noalloc(dx, dwq, ds, dz)
        y_ws = C.gemv(dx, dwq, ds, dz)
        torch.cuda.synchronize()
        torch.testing.assert_close(y_na.float(), y_ws.float(), atol=ATOL, rtol=RTOL)
        ref = ow.bf16_to_f32(ow.linear(x, wq, s, z))
        np.testing.assert_allclose(y_na.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
        outs.append(y_na)
    # the second call did not disturb the first call's result
    assert not torch.equal(outs[0], outs[1])


class _DevBytes:
    """A zero-copy uint8 view of device memory at `ptr` (for reading the scratch)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def test_noalloc_leaves_scratch_zero(cuda):
    """Every call leaves the scratch all zero again, including shapes whose row
    blocks are split across CTAs and finished through partial words in the
    scratch (K=8192, N=11008 and K=4096, N=28672 at M=8)."""
    import ctypes

    for (M, K, N) in [(8, 8192, 11008), (8, 4096, 28672), (1, 4096, 4096)]:
        x, wq, s, z = ow.baseline_case(M, K, N, seed=77)
        noalloc(C.to_dev_bf16(x, cuda), C.to_dev(wq, cuda), C.to_dev(s, cuda), C.to_dev(z, cuda))
    torch.cuda.synchronize()
    ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
    _lib.call("focal_w4a16_noalloc_scratch", ctypes.byref(ptr), ctypes.byref(nbytes))
    assert nbytes.value == 8 << 20
    scratch = torch.as_tensor(_DevBytes(ptr.value, nbytes.value), device=cuda)
    assert int(scratch.count_nonzero()) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda, monkeypatch):
    """A shape whose workspace bound exceeds the scratch is refused with
    FOCAL_ERR_UNSUPPORTED and a message that names the limit.  No contract shape
    reaches the 8 MiB on a 148-SM B200, so the limit is lowered through the
    library's test hook."""
    monkeypatch.setenv("FOCAL_W4A16_NOALLOC_LIMIT", "4096")
    x, wq, s, z = ow.baseline_case(1, 4096, 4096, seed=78)
    with pytest.raises(_lib.FocalError) as e:
        noalloc(C.to_dev_bf16(x, cuda), C.to_dev(wq, cuda), C.to_dev(s, cuda), C.to_dev(z, cuda))
    assert e.value.code == _lib.FOCAL_ERR_UNSUPPORTED
    assert "scratch" in str(e.value) and "4096" in str(e.value)
