"""Test helpers: call the C ABI (include/focal_b200.h) on torch device tensors,
and move tensors between torch and the numpy oracle's bit-pattern format."""
from __future__ import annotations

import numpy as np
import torch

from focal_b200 import _lib


def stream_ptr():
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def to_dev_bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_dev(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def w4a16_workspace(M, K, N, device):
    """A fresh workspace: zeroed, as the C ABI requires before its first use."""
    n = int(_lib.lib().focal_w4a16_workspace_size(M, K, N))
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device), n


def gemv(x, wq, scales, zeros, out_dtype=torch.bfloat16, ws=None):
    M, K = x.shape
    N = wq.shape[0]
    y = torch.empty((M, N), dtype=out_dtype, device=x.device)
    buf, n = ws if ws is not None else w4a16_workspace(M, K, N, x.device)
    name = "focal_w4a16_gemv" if out_dtype == torch.bfloat16 else "focal_w4a16_gemv_f32"
    _lib.call(name, ptr(x), ptr(wq), ptr(scales), ptr(zeros), ptr(y), M, K, N, ptr(buf), n, stream_ptr())
    return y


def gate_up_silu(x, gate, up):
    M, K = x.shape
    N = gate[0].shape[0]
    h = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    buf, n = w4a16_workspace(M, K, N, x.device)
    _lib.call("focal_w4a16_gate_up_silu", ptr(x), *map(ptr, gate), *map(ptr, up), ptr(h), M, K, N,
              ptr(buf), n, stream_ptr())
    return h


def dequant(wq, scales, zeros, K):
    N = wq.shape[0]
    w = torch.empty((N, K), dtype=torch.float32, device=wq.device)
    _lib.call("focal_w4a16_dequant", ptr(wq), ptr(scales), ptr(zeros), ptr(w), K, N, stream_ptr())
    return w


def pack(q):
    N, K = q.shape
    wq = torch.empty((N, K // 8), dtype=torch.int32, device=q.device)
    _lib.call("focal_pack_int4", ptr(q), ptr(wq), N, K, stream_ptr())
    return wq


def attention_workspace(B, Hq, Hkv, L, D, device):
    n = _lib.lib().focal_gqa_decode_workspace_size(B, Hq, Hkv, L, D)
    return torch.zeros(max(int(n), 256), dtype=torch.uint8, device=device), int(n)


def attention(q, k, v, scale=None, ws=None):
    B, Hq, D = q.shape
    Hkv, L = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    if ws is None:
        ws = attention_workspace(B, Hq, Hkv, L, D, q.device)
    buf, n = ws
    o = torch.empty_like(q)
    _lib.call("focal_gqa_decode_attn", ptr(q), ptr(k), ptr(v), ptr(o), B, Hq, Hkv, L, D,
              float(scale), ptr(buf), n, stream_ptr())
    return o


def tile_pack(wq, scales, zeros):
    N, K = wq.shape[0], wq.shape[1] * 8
    t = torch.empty(int(_lib.lib().focal_w4a16_tiles_size(K, N)), dtype=torch.uint8, device=wq.device)
    _lib.call("focal_w4a16_tile_pack", ptr(wq), ptr(scales), ptr(zeros), ptr(t), K, N, stream_ptr())
    return t


def tile_unpack(t, K, N):
    wq = torch.empty((N, K // 8), dtype=torch.int32, device=t.device)
    s = torch.empty((N, K // 128), dtype=torch.float16, device=t.device)
    z = torch.empty((N, K // 128), dtype=torch.float16, device=t.device)
    _lib.call("focal_w4a16_tile_unpack", ptr(t), ptr(wq), ptr(s), ptr(z), K, N, stream_ptr())
    return wq, s, z


def gemv_tiled(x, tiles, N, out_dtype=torch.bfloat16):
    M, K = x.shape
    y = torch.empty((M, N), dtype=out_dtype, device=x.device)
    buf, n = w4a16_workspace(M, K, N, x.device)
    name = "focal_w4a16_gemv_tiled" if out_dtype == torch.bfloat16 else "focal_w4a16_gemv_tiled_f32"
    _lib.call(name, ptr(x), ptr(tiles), ptr(y), M, K, N, ptr(buf), n, stream_ptr())
    return y


def gate_up_silu_tiled(x, tiles_gate, tiles_up, N):
    M, K = x.shape
    h = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    buf, n = w4a16_workspace(M, K, N, x.device)
    _lib.call("focal_w4a16_gate_up_silu_tiled", ptr(x), ptr(tiles_gate), ptr(tiles_up), ptr(h), M, K, N,
              ptr(buf), n, stream_ptr())
    return h


def paged_attention(q, k_pages, v_pages, block_table, seq_lens, max_seq_len, scale=None, ws=None):
    B, Hq, D = q.shape
    num_pages, Hkv, page_size = k_pages.shape[0], k_pages.shape[1], k_pages.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    if ws is None:
        ws = attention_workspace(B, Hq, Hkv, max_seq_len, D, q.device)
    buf, n = ws
    o = torch.empty_like(q)
    _lib.call("focal_gqa_decode_paged", ptr(q), ptr(k_pages), ptr(v_pages), ptr(block_table), ptr(seq_lens),
              ptr(o), B, Hq, Hkv, D, num_pages, page_size, block_table.shape[1], max_seq_len, float(scale),
              ptr(buf), n, stream_ptr())
    return o
