"""The attention oracle is unpinned by the reference (which has no attention);
cross-check it against torch's CPU scaled_dot_product_attention instead."""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import w4a16 as ow


@pytest.mark.parametrize("B,Hq,Hkv,L", [(1, 32, 8, 64), (2, 32, 8, 129), (1, 8, 8, 17), (2, 16, 2, 40)])
def test_oracle_matches_torch_sdpa(B, Hq, Hkv, L):
    D = 128
    q, k, v = oa.random_case(B, Hq, Hkv, L, D, seed=7 + L)
    o = oa.decode_attention(q, k, v, out="f64")
    qt = torch.from_numpy(ow.bf16_to_f32(q)).double().unsqueeze(2)          # [B,Hq,1,D]
    kt = torch.from_numpy(ow.bf16_to_f32(k)).double().repeat_interleave(Hq // Hkv, dim=1)
    vt = torch.from_numpy(ow.bf16_to_f32(v)).double().repeat_interleave(Hq // Hkv, dim=1)
    ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt).squeeze(2).numpy()
    assert np.allclose(o, ref, atol=1e-12, rtol=1e-10)


def test_oracle_single_position_returns_v():
    q, k, v = oa.random_case(1, 4, 1, 1, 128, seed=3)
    o = oa.decode_attention(q, k, v)
    assert np.array_equal(o, np.repeat(v[:, :, 0, :], 4, axis=1))


def _pages(k, page_size, seed):
    """Scatter k [B, Hkv, L, D] into shuffled pages; return (pages, block table)."""
    B, Hkv, L, D = k.shape
    per = -(-L // page_size)
    order = np.random.default_rng(seed).permutation(B * per + 2)
    pages = np.zeros((B * per + 2, Hkv, page_size, D), dtype=k.dtype)
    table = np.zeros((B, per), dtype=np.int32)
    for b in range(B):
        for j in range(per):
            rows = min(page_size, L - j * page_size)
            pages[order[b * per + j], :, :rows] = k[b, :, j * page_size: j * page_size + rows]
            table[b, j] = order[b * per + j]
    return pages, table


@pytest.mark.parametrize("page_size", [16, 64])
def test_paged_oracle_equals_contiguous(page_size):
    q, k, v = oa.random_case(3, 8, 2, 100, 128, seed=page_size)
    kp, table = _pages(k, page_size, seed=1)
    vp, _ = _pages(v, page_size, seed=1)
    full = oa.decode_attention_paged(q, kp, vp, table, np.array([100, 100, 100]))
    assert np.array_equal(full, oa.decode_attention(q, k, v))
    ragged = oa.decode_attention_paged(q, kp, vp, table, np.array([1, 37, 100]))
    for b, L in enumerate((1, 37, 100)):
        want = oa.decode_attention(q[b:b + 1], k[b:b + 1, :, :L], v[b:b + 1, :, :L])
        assert np.array_equal(ragged[b:b + 1], want)
