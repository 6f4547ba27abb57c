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
