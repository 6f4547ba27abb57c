"""numpy restatement of contiguous GQA decode attention — TEST INFRASTRUCTURE ONLY.

Parity UNPINNED: the reference project has no attention code (its
bench/bench_decode_bundle.py:19-27 times projections only), so this oracle is
written from the mathematics of scaled dot-product attention and cross-checked
against torch's CPU ``scaled_dot_product_attention`` in
tests/test_oracle_attention.py.

Contract (defined by this project):
    q [B, Hq, D], k/v [B, Hkv, L, D] (bf16 bit patterns as uint16),
    query head h reads KV head h // (Hq // Hkv)  (the usual ``repeat_kv`` grouping),
    o[b, h] = softmax(q[b, h] . k[b, g]^T * scale) . v[b, g]
computed in float64 here (fp32 on the GPU) and rounded to bf16.
"""
from __future__ import annotations

import numpy as np

from .w4a16 import bf16_to_f32, f32_to_bf16


def decode_attention(q_bf16: np.ndarray, k_bf16: np.ndarray, v_bf16: np.ndarray,
                     scale: float | None = None, out: str = "bf16") -> np.ndarray:
    q = bf16_to_f32(q_bf16).astype(np.float64)
    k = bf16_to_f32(k_bf16).astype(np.float64)
    v = bf16_to_f32(v_bf16).astype(np.float64)
    B, Hq, D = q.shape
    Bk, Hkv, L, Dk = k.shape
    if Bk != B or Dk != D or v.shape != k.shape or Hq % Hkv != 0:
        raise ValueError("shape mismatch")
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    grp = Hq // Hkv
    qg = q.reshape(B, Hkv, grp, D)
    s = np.einsum("bhgd,bhld->bhgl", qg, k) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhgl,bhld->bhgd", p, v).reshape(B, Hq, D)
    if out == "f64":
        return o
    return f32_to_bf16(o.astype(np.float32))


def random_case(B: int, Hq: int, Hkv: int, L: int, D: int, seed: int):
    """q, k, v ~ N(0,1) rounded to bf16 bits (the benchmark's distribution)."""
    rng = np.random.default_rng(seed)
    q = f32_to_bf16(rng.standard_normal((B, Hq, D), dtype=np.float32))
    k = f32_to_bf16(rng.standard_normal((B, Hkv, L, D), dtype=np.float32))
    v = f32_to_bf16(rng.standard_normal((B, Hkv, L, D), dtype=np.float32))
    return q, k, v


def paged_to_contiguous(pages: np.ndarray, block_table: np.ndarray, b: int, L: int) -> np.ndarray:
    """Sequence b's first L positions gathered from pages [num_pages, Hkv,
    page_size, D] through its block-table row: [Hkv, L, D]."""
    page_size = pages.shape[2]
    n = (L + page_size - 1) // page_size
    seq = np.concatenate([pages[block_table[b, j]] for j in range(n)], axis=1)
    return seq[:, :L]


def decode_attention_paged(q_bf16: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                           block_table: np.ndarray, seq_lens: np.ndarray, scale: float | None = None) -> np.ndarray:
    """Paged, variable-length decode attention: each sequence b attends over its
    own seq_lens[b] positions, read page by page through its block-table row
    (the same mathematics as decode_attention, one sequence at a time)."""
    out = []
    for b in range(q_bf16.shape[0]):
        L = int(seq_lens[b])
        k = paged_to_contiguous(k_pages, block_table, b, L)[None]
        v = paged_to_contiguous(v_pages, block_table, b, L)[None]
        out.append(decode_attention(q_bf16[b:b + 1], k, v, scale)[0])
    return np.stack(out)
