"""focal_b200 — B200-native (sm_100a) decode hot paths of focal-w4a16.

Drop-in for the reference package's API (focal_w4a16/__init__.py:6-133 in the
reference project): the same names, argument meaning, packing layout and error
types, with the arithmetic in hand-written sm_100a kernels (libfocal_b200.so,
C ABI in include/focal_b200.h) reached through a thin PyTorch extension
(focal_b200._C).  There is no CPU or library fallback: every entry point
raises if the extension is missing.

Reference API mirrored here:
    w4a16_linear, pack_int4_weight, dequant_ref, random_case,
    require_cuda_contiguous, SUPPORTED_M/K/N/EXTRA_SHAPES
Added for the decode paths this package also covers:
    w4a16_linear_f32, w4a16_gate_up_silu, decode_mlp, gqa_decode_attention,
    baseline_case, check_shape
"""
from __future__ import annotations

from importlib import import_module

import torch

# The reference's validated shape whitelist (focal_w4a16/__init__.py:6-14).
# The kernels here accept the wider rule-based contract of check_shape().
SUPPORTED_M = (1, 2, 4, 8)
SUPPORTED_K = (4096, 8192)
SUPPORTED_N = (4096, 8192, 11008)
SUPPORTED_EXTRA_SHAPES = tuple((m, 11008, 4096) for m in SUPPORTED_M)

GROUP_SIZE = 128
extension = None


def _ext():
    """Import the PyTorch extension on first use (as the reference does,
    focal_w4a16/__init__.py:25-27), after loading the C-ABI library it links."""
    global extension
    if extension is None:
        from . import _lib

        _lib.lib()
        extension = import_module("focal_b200._C")
    return extension


# ------------------------------------------------------------------ W4A16
def w4a16_linear(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                 zeros: torch.Tensor) -> torch.Tensor:
    """y[M, N] = bf16(x[M, K] @ dequant(wq, scales, zeros)[N, K]^T), fp32 accumulation.

    Same contract as the reference (focal_w4a16/__init__.py:18-28): CUDA,
    contiguous inputs of dtypes bf16 / int32 / fp16 / fp16; the bf16 output is
    allocated on x's device and computed on the current stream; violations
    raise RuntimeError with the reference's messages.
    """
    return _ext().w4a16_linear(x, wq, scales, zeros)


def w4a16_linear_f32(x, wq, scales, zeros) -> torch.Tensor:
    """As w4a16_linear but returns the fp32 sums unrounded (row-parallel partials)."""
    return _ext().w4a16_linear_f32(x, wq, scales, zeros)


def w4a16_gate_up_silu(x, gate, up) -> torch.Tensor:
    """h = bf16(silu(bf16(x Wg^T)) * bf16(x Wu^T)) in one kernel; gate/up are
    (wq, scales, zeros) triples of the same shape."""
    return _ext().w4a16_gate_up_silu(x, *gate, *up)


def decode_mlp(x, gate, up, down) -> torch.Tensor:
    """Llama-style decode MLP: down(silu(gate(x)) * up(x)), all W4A16."""
    return w4a16_linear(w4a16_gate_up_silu(x, gate, up), *down)


def w4a16_tile_pack(wq: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor) -> torch.Tensor:
    """Offline re-layout of (wq, scales, zeros) into unit-tiled weights: a flat
    uint8 tensor, one contiguous 8704-byte chunk per 64 rows x 256 K values
    (include/focal_b200.h).  The linears below give the same bits on it as
    their reference-layout counterparts on the original weights."""
    return _ext().tile_pack(wq, scales, zeros)


def w4a16_linear_tiled(x: torch.Tensor, tiles: torch.Tensor, N: int) -> torch.Tensor:
    """w4a16_linear on unit-tiled weights (N output rows)."""
    return _ext().w4a16_linear_tiled(x, tiles, N)


def w4a16_linear_tiled_f32(x: torch.Tensor, tiles: torch.Tensor, N: int) -> torch.Tensor:
    """w4a16_linear_f32 on unit-tiled weights."""
    return _ext().w4a16_linear_tiled_f32(x, tiles, N)


def w4a16_gate_up_silu_tiled(x: torch.Tensor, tiles_gate: torch.Tensor, tiles_up: torch.Tensor,
                             N: int) -> torch.Tensor:
    """w4a16_gate_up_silu on unit-tiled gate and up weights."""
    return _ext().w4a16_gate_up_silu_tiled(x, tiles_gate, tiles_up, N)


def check_shape(M: int, K: int, N: int) -> None:
    """Raise RuntimeError (reference wording) if (M, K, N) is outside the contract."""
    from . import _lib

    rc = _lib.lib().focal_w4a16_check_shape(int(M), int(K), int(N))
    if rc != 0:
        raise RuntimeError(_lib.last_error())


def require_cuda_contiguous(name: str, tensor: torch.Tensor) -> None:
    if not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def pack_int4_weight(w_q_uint8: torch.Tensor) -> torch.Tensor:
    """uint8 [N, K] -> int32 [N, K/8], value k at bits 4*(k % 8) of word k // 8
    (reference focal_w4a16/__init__.py:38-54; packed on the GPU here)."""
    require_cuda_contiguous("w_q_uint8", w_q_uint8)
    if w_q_uint8.dtype != torch.uint8:
        raise ValueError("w_q_uint8 must have dtype torch.uint8")
    if w_q_uint8.ndim != 2:
        raise ValueError("w_q_uint8 must have shape [N, K]")
    if w_q_uint8.shape[1] % 8 != 0:
        raise ValueError("K must be divisible by 8")
    return _ext().pack_int4(w_q_uint8)


def dequant_ref(wq: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, K: int) -> torch.Tensor:
    """fp32 [N, K] = (q - zeros) * scales per 128-wide group, bit-identical to the
    reference (focal_w4a16/__init__.py:57-91); computed by a CUDA kernel here."""
    require_cuda_contiguous("wq", wq)
    require_cuda_contiguous("scales", scales)
    require_cuda_contiguous("zeros", zeros)
    if wq.dtype != torch.int32:
        raise ValueError("wq must have dtype torch.int32")
    if scales.dtype != torch.float16:
        raise ValueError("scales must have dtype torch.float16")
    if zeros.dtype != torch.float16:
        raise ValueError("zeros must have dtype torch.float16")
    if wq.ndim != 2:
        raise ValueError("wq must have shape [N, K / 8]")
    if K % GROUP_SIZE != 0:
        raise ValueError("K must be divisible by 128")
    n, k_words = wq.shape
    if k_words * 8 != K:
        raise ValueError("wq shape does not match K")
    if tuple(scales.shape) != (n, K // GROUP_SIZE):
        raise ValueError("scales must have shape [N, K / 128]")
    if tuple(zeros.shape) != (n, K // GROUP_SIZE):
        raise ValueError("zeros must have shape [N, K / 128]")
    return _ext().dequant(wq, scales, zeros, K)


def random_case(M: int, K: int, N: int, seed: int):
    """The reference's test-case generator (focal_w4a16/__init__.py:94-121):
    the same shape whitelist and the same CUDA-generator draws in the same
    order, so a seed gives the reference's exact tensors."""
    if M not in SUPPORTED_M:
        raise ValueError(f"unsupported M: {M}")
    if K not in SUPPORTED_K and (M, K, N) not in SUPPORTED_EXTRA_SHAPES:
        raise ValueError(f"unsupported shape: M={M} K={K} N={N}")
    if N not in SUPPORTED_N:
        raise ValueError(f"unsupported N: {N}")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required")
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    opts = dict(device="cuda", generator=gen)
    x = torch.randn((M, K), dtype=torch.bfloat16, **opts)
    nibbles = torch.randint(0, 16, (N, K), dtype=torch.uint8, **opts)
    wq = pack_int4_weight(nibbles)
    scales = 0.005 + 0.045 * torch.rand((N, K // GROUP_SIZE), dtype=torch.float16, **opts)
    zeros = 7.0 + torch.rand((N, K // GROUP_SIZE), dtype=torch.float16, **opts)
    return x.contiguous(), wq, scales.contiguous(), zeros.contiguous()


def baseline_case(M: int, K: int, N: int, seed: int, device="cuda"):
    """Benchmark inputs: x ~ N(0,1) bf16; wq uniform random 32-bit words; scales
    fp16 U[0.005, 0.02]; zeros fp16 integers 0..15.  Drawn on a seeded CPU
    generator (identical on every machine), then moved to `device`."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((M, K), generator=g, dtype=torch.float32).to(torch.bfloat16)
    wq = torch.randint(-(2**31), 2**31, (N, K // 8), generator=g, dtype=torch.int64).to(torch.int32)
    scales = (0.005 + 0.015 * torch.rand((N, K // GROUP_SIZE), generator=g)).to(torch.float16)
    zeros = torch.randint(0, 16, (N, K // GROUP_SIZE), generator=g, dtype=torch.int64).to(torch.float16)
    return tuple(t.to(device).contiguous() for t in (x, wq, scales, zeros))


# ------------------------------------------------------------ attention
def gqa_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         scale: float | None = None) -> torch.Tensor:
    """Decode attention over a contiguous KV cache.

    q [B, Hq, D] bf16 (one token per sequence); k_cache / v_cache
    [B, Hkv, L, D] bf16; query head h attends KV head h // (Hq // Hkv);
    scale defaults to 1/sqrt(D).  Returns o [B, Hq, D] bf16.  D must be 128.
    """
    return _ext().gqa_decode_attention(q, k_cache, v_cache, scale)


def gqa_decode_attention_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                               block_table: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int,
                               scale: float | None = None) -> torch.Tensor:
    """Decode attention over a paged KV cache with per-sequence lengths.

    k_pages / v_pages [num_pages, Hkv, page_size, D] bf16 (page_size 16, 32 or
    a multiple of 64); block_table int32 [B, max_pages] maps page j of
    sequence b to a page; seq_lens int32 [B] in 1..max_seq_len.  max_seq_len
    (a host integer, an upper bound on seq_lens) sizes the launch.  Returns
    o [B, Hq, D] bf16.
    """
    return _ext().gqa_decode_attention_paged(q, k_pages, v_pages, block_table, seq_lens, max_seq_len, scale)


__all__ = [
    "SUPPORTED_K",
    "SUPPORTED_M",
    "SUPPORTED_N",
    "SUPPORTED_EXTRA_SHAPES",
    "baseline_case",
    "check_shape",
    "decode_mlp",
    "dequant_ref",
    "gqa_decode_attention",
    "gqa_decode_attention_paged",
    "pack_int4_weight",
    "random_case",
    "require_cuda_contiguous",
    "w4a16_gate_up_silu",
    "w4a16_linear",
    "w4a16_linear_f32",
]
