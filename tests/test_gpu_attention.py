"""GQA decode attention parity on the GPU, through the C ABI, against the
float64 numpy oracle (oracle/attention.py; parity unpinned by the reference,
which has no attention).  Bar: allclose atol 2e-2 / rtol 1e-2 after the bf16
cast, plus a relative-L2 error below 1e-2 (bf16 P and output rounding)."""
import numpy as np
import pytest
import torch

import focal_b200
from oracle import attention as oa
from oracle import w4a16 as ow
from tests import _capi as C

pytestmark = pytest.mark.gpu


def check(o_dev, q, k, v, what):
    ref = oa.decode_attention(q, k, v, out="f64")
    got = ow.bf16_to_f32(C.bf16_bits(o_dev)).astype(np.float64)
    rel_l2 = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert np.allclose(got, ref, atol=2e-2, rtol=1e-2), (what, np.abs(got - ref).max())
    assert rel_l2 < 1e-2, (what, rel_l2)
    return rel_l2


def run(B, Hq, Hkv, L, seed, device):
    q, k, v = oa.random_case(B, Hq, Hkv, L, 128, seed)
    o = C.attention(C.to_dev_bf16(q, device), C.to_dev_bf16(k, device), C.to_dev_bf16(v, device))
    return check(o, q, k, v, f"B={B} Hq={Hq} Hkv={Hkv} L={L}")


@pytest.mark.parametrize("B,Hq,Hkv,L", [
    (1, 32, 8, 1), (1, 32, 8, 5), (1, 32, 8, 64), (1, 32, 8, 65), (2, 32, 8, 200),
    (1, 8, 8, 100), (1, 16, 8, 300), (1, 64, 4, 130), (3, 32, 2, 1000), (1, 32, 32, 77),
])
def test_small_and_ragged(cuda, B, Hq, Hkv, L):
    run(B, Hq, Hkv, L, seed=B * 1000 + L, device=cuda)


@pytest.mark.parametrize("B", [1, 4, 8])
@pytest.mark.parametrize("L", [512, 4096, 32768])
def test_contract_shapes(cuda, B, L):
    run(B, 32, 8, L, seed=7 * B + L, device=cuda)


def test_workspace_counters_left_zero_and_repeatable(cuda):
    q, k, v = oa.random_case(2, 32, 8, 4096, 128, seed=3)
    dq, dk, dv = (C.to_dev_bf16(a, cuda) for a in (q, k, v))
    ws = C.attention_workspace(2, 32, 8, 4096, 128, cuda)
    o1 = C.attention(dq, dk, dv, ws=ws)
    torch.cuda.synchronize()
    assert int(ws[0][:64].sum()) == 0  # per-(b, kv head) counters
    o2 = C.attention(dq, dk, dv, ws=ws)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_public_api_and_scale(cuda):
    q, k, v = oa.random_case(2, 32, 8, 777, 128, seed=11)
    dq, dk, dv = (C.to_dev_bf16(a, cuda) for a in (q, k, v))
    o = focal_b200.gqa_decode_attention(dq, dk, dv)
    check(o, q, k, v, "api")
    o2 = focal_b200.gqa_decode_attention(dq, dk, dv, scale=0.05)
    ref = oa.decode_attention(q, k, v, scale=0.05, out="f64")
    got = ow.bf16_to_f32(C.bf16_bits(o2)).astype(np.float64)
    assert np.allclose(got, ref, atol=2e-2, rtol=1e-2)
    with pytest.raises(RuntimeError, match="head_dim"):
        focal_b200.gqa_decode_attention(dq[..., :64].contiguous(), dk[..., :64].contiguous(),
                                        dv[..., :64].contiguous())


def test_capi_workspace_too_small(cuda):
    from focal_b200 import _lib

    q, k, v = (C.to_dev_bf16(a, cuda) for a in oa.random_case(1, 32, 8, 4096, 128, seed=1))
    o = torch.empty_like(q)
    rc = _lib.lib().focal_gqa_decode_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                          1, 32, 8, 4096, 128, 0.088, None, 0, C.stream_ptr())
    assert rc == _lib.FOCAL_ERR_WORKSPACE


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("B,L", [(1, 4096), (4, 700)])
def test_head_sharded_attention(cuda, world, B, L):
    """Tensor parallelism over KV heads (focal_b200.tp.heads_shard and
    HeadParallelAttention), its ranks run in turn on one GPU: each rank's
    shard of q and of the caches goes through the kernel, and the shards'
    outputs joined in rank order (what gather_heads' all-gather does) match
    the oracle on the full heads, and the unsharded kernel's output within
    one bf16 step (the split plan depends on the number of heads)."""
    from focal_b200 import tp

    q, k, v = oa.random_case(B, 32, 8, L, 128, seed=40 + world)
    dq, dk, dv = (C.to_dev_bf16(a, cuda) for a in (q, k, v))
    parts = []
    for rank in range(world):
        ql, kl, vl = tp.heads_shard(dq, dk, dv, rank, world)
        parts.append(tp.HeadParallelAttention()(ql, kl, vl))  # one-rank group: the shard's own output
    o = torch.cat(parts, dim=1)
    assert o.shape == (B, 32, 128)
    check(o, q, k, v, f"heads world={world} B={B} L={L}")
    full = focal_b200.gqa_decode_attention(dq, dk, dv)
    diff = (o.float() - full.float()).abs()
    assert float((diff / full.float().abs().clamp_min(1.0)).max()) <= 2 ** -7
