"""CPU-only checks of the native boundary: the C-ABI library loads without a
GPU, exports every entry point include/focal_b200.h declares, and its
host-only functions (shape contract, workspace sizing) behave."""
import ctypes
import re
from pathlib import Path

import pytest

from focal_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "focal_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(focal_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "focal_w4a16_gemv" in names and "focal_gqa_decode_attn" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert L.focal_abi_version() == 1


@pytest.mark.parametrize("M,K,N,msg", [
    (1, 4096, 4096, None), (8, 11008, 4096, None), (3, 8192, 28672, None), (8, 28672, 8192, None),
    (0, 4096, 4096, "unsupported M"), (9, 4096, 4096, "unsupported M"),
    (1, 4096, 4100, "unsupported N"), (1, 4096, 0, "unsupported N"),
    (1, 11008, 11008, "unsupported K/N"), (1, 4224, 4096, "unsupported K/N"),
    (1, 100, 4096, "unsupported K/N"), (8, 40960, 4096, None), (1, 1 << 25, 64, "unsupported K/N"),
    (1, 4096, 262144, None), (1, 4096, 262144 + 64, "unsupported N"),
])
def test_shape_contract(M, K, N, msg):
    rc = _lib.lib().focal_w4a16_check_shape(M, K, N)
    if msg is None:
        assert rc == _lib.FOCAL_OK
    else:
        assert rc == _lib.FOCAL_ERR_UNSUPPORTED and _lib.last_error() == msg


def test_w4a16_workspace_sizing():
    L = _lib.lib()
    # 16 KB of row-block counters at a fixed place, then split partials, whose
    # number depends on M (tokens per partial) and on how many ranges split
    # the row blocks, not on K
    a = L.focal_w4a16_workspace_size(1, 4096, 4096)
    b = L.focal_w4a16_workspace_size(8, 4096, 4096)
    c = L.focal_w4a16_workspace_size(8, 8192, 4096)
    assert a >= 16384 and a % 256 == 0
    assert a < b <= c
    assert L.focal_w4a16_workspace_size(9, 4096, 4096) == 0
    assert L.focal_w4a16_workspace_size(1, 4096, 100) == 0
    assert L.focal_w4a16_workspace_size(1, 4096, 262144 + 64) == 0


def test_attention_workspace_sizing():
    L = _lib.lib()
    small = L.focal_gqa_decode_workspace_size(1, 32, 8, 512, 128)
    big = L.focal_gqa_decode_workspace_size(8, 32, 8, 32768, 128)
    assert 0 < small < big
    assert L.focal_gqa_decode_workspace_size(1, 32, 8, 512, 64) == 0  # unsupported head dim
    assert L.focal_gqa_decode_workspace_size(1, 30, 8, 512, 128) == 0  # Hq % Hkv != 0


def test_status_codes_have_messages_without_gpu():
    L = _lib.lib()
    # argument errors are caught on the host before any CUDA call
    rc = L.focal_w4a16_gemv(None, None, None, None, None, 1, 4096, 4096, None, 0, None)
    assert rc == _lib.FOCAL_ERR_INVALID_VALUE and "null" in _lib.last_error()
    rc = L.focal_pack_int4(None, None, 4, 12, None)
    assert rc == _lib.FOCAL_ERR_UNSUPPORTED
    with pytest.raises(_lib.FocalError, match="unsupported M"):
        _lib.call("focal_w4a16_check_shape", 16, 4096, 4096)
    assert isinstance(ctypes.c_int(0).value, int)


def test_tp_buffer_sizing_and_argument_errors():
    L = _lib.lib()
    one = L.focal_tp_buffer_size(1, 8, 4096)
    two = L.focal_tp_buffer_size(2, 8, 4096)
    # 256 B of state, then two receive halves of world x M x N 8-byte
    # {payload, epoch} words
    assert one == 256 + 2 * 1 * 8 * 4096 * 8
    assert two - one == 2 * 8 * 4096 * 8
    assert L.focal_tp_buffer_size(9, 8, 4096) == 0
    assert L.focal_tp_buffer_size(2, 9, 4096) == 0
    assert L.focal_tp_buffer_size(2, 8, 100) == 0
    for name in ("focal_w4a16_gemv_allgather", "focal_w4a16_gemv_allreduce"):
        rc = getattr(L, name)(None, None, None, None, None, 8, 4096, 4096, None, None, 0, None)
        assert rc == _lib.FOCAL_ERR_INVALID_VALUE and "null tensor-parallel group" in _lib.last_error()
    comm = _lib.TpComm()
    comm.world, comm.rank, comm.bytes = 2, 1, two
    rc = L.focal_w4a16_gemv_allreduce(None, None, None, None, None, 8, 4096, 4096, ctypes.byref(comm),
                                      None, 0, None)
    assert rc == _lib.FOCAL_ERR_INVALID_VALUE and "rank 0 is null" in _lib.last_error()


def test_paged_attention_argument_errors_without_gpu():
    L = _lib.lib()
    args = dict(B=2, Hq=32, Hkv=8, D=128, num_pages=16, page_size=24, max_pages=8, max_len=128)

    def call(**kw):
        a = dict(args, **kw)
        return L.focal_gqa_decode_paged(None, None, None, None, None, None, a["B"], a["Hq"], a["Hkv"], a["D"],
                                        a["num_pages"], a["page_size"], a["max_pages"], a["max_len"], 0.1,
                                        None, 0, None)

    assert call() == _lib.FOCAL_ERR_UNSUPPORTED and "page_size" in _lib.last_error()
    assert call(page_size=16, max_pages=4) == _lib.FOCAL_ERR_UNSUPPORTED and "max_seq_len" in _lib.last_error()
    assert call(page_size=64, D=64) == _lib.FOCAL_ERR_UNSUPPORTED and "head_dim" in _lib.last_error()
    assert call(page_size=128) == _lib.FOCAL_ERR_INVALID_VALUE and "null" in _lib.last_error()

def test_reference_extension_module_name_resolves():
    """`import focal_w4a16._C` (the module the reference package imports) loads
    the B200 extension and exposes its entry points; no GPU is touched."""
    import importlib

    m = importlib.import_module("focal_w4a16._C")
    for name in ("w4a16_linear", "w4a16_linear_f32", "w4a16_gate_up_silu", "gqa_decode_attention"):
        assert callable(getattr(m, name)), name
