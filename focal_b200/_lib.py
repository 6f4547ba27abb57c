"""ctypes binding of the C ABI in include/focal_b200.h (libfocal_b200.so).

This is the binding a non-PyTorch host would write; the parity tests and the
end-to-end benchmark leg call the kernels through it.  Loading fails loudly if
the library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfocal_b200.so"

FOCAL_OK = 0
FOCAL_ERR_INVALID_VALUE = 1
FOCAL_ERR_UNSUPPORTED = 2
FOCAL_ERR_WORKSPACE = 3
FOCAL_ERR_CUDA = 4
FOCAL_ERR_DEVICE = 5

_P = ctypes.c_void_p
_I = ctypes.c_int
_S = ctypes.c_size_t
_F = ctypes.c_float


class TpComm(ctypes.Structure):
    """struct focal_tp_comm: every rank's buffer as mapped in this process."""

    _fields_ = [("peer", ctypes.c_void_p * 8), ("bytes", ctypes.c_size_t),
                ("world", ctypes.c_int), ("rank", ctypes.c_int)]


_C = ctypes.POINTER(TpComm)

# name -> (restype, argtypes); mirrors include/focal_b200.h
SIGNATURES = {
    "focal_last_error": (ctypes.c_char_p, []),
    "focal_abi_version": (_I, []),
    "focal_w4a16_check_shape": (_I, [_I, _I, _I]),
    "focal_w4a16_workspace_size": (_S, [_I, _I, _I]),
    "focal_w4a16_gemv": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_w4a16_gemv_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "focal_w4a16_noalloc_scratch": (_I, [ctypes.POINTER(_P), ctypes.POINTER(_S)]),
    "focal_w4a16_gemv_f32": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_w4a16_gate_up_silu": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_w4a16_tiles_size": (_S, [_I, _I]),
    "focal_w4a16_tile_pack": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "focal_w4a16_tile_unpack": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "focal_w4a16_gemv_tiled": (_I, [_P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_w4a16_gemv_tiled_f32": (_I, [_P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_w4a16_gate_up_silu_tiled": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _S, _P]),
    "focal_tp_buffer_size": (_S, [_I, _I, _I]),
    "focal_tp_buffer_create": (_I, [_S, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_uint8)]),
    "focal_tp_buffer_open": (_I, [ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(_P)]),
    "focal_tp_buffer_close": (_I, [_P]),
    "focal_tp_buffer_destroy": (_I, [_P]),
    "focal_w4a16_gemv_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _C, _P, _S, _P]),
    "focal_w4a16_gemv_allreduce": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _C, _P, _S, _P]),
    "focal_w4a16_dequant": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "focal_pack_int4": (_I, [_P, _P, _I, _I, _P]),
    "focal_gqa_decode_workspace_size": (_S, [_I, _I, _I, _I, _I]),
    "focal_gqa_decode_attn": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _S, _P]),
    "focal_gqa_decode_paged": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _S, _P]),
    "focal_device_status": (_I, [ctypes.POINTER(_I)]),
    "focal_device_status_peek": (_I, [ctypes.POINTER(_I)]),
    "focal_reset_device_status": (_I, []),
}

_lib = None


class FocalError(RuntimeError):
    """A focal_b200 C-ABI call returned a nonzero focal_status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libfocal_b200.so once (RTLD_GLOBAL, so the PyTorch extension that
    links against it resolves to this copy)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m focal_b200.build` "
                "(focal_b200 has no non-CUDA fallback)")
        handle = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().focal_last_error().decode()


def check(rc: int) -> None:
    if rc != FOCAL_OK:
        raise FocalError(rc, last_error())


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise FocalError on failure."""
    check(getattr(lib(), name)(*args))
