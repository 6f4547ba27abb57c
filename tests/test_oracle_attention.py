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
