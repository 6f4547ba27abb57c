"""Paged, variable-length GQA decode attention (focal_gqa_decode_paged) on
the GPU, through the C ABI.

Bars: pages holding the contiguous caches in a shuffled order, with every
sequence at full length, give the contiguous kernel's bits exactly (same
plan, same arithmetic), even when the unused rows of the last pages hold
NaN; variable lengths match the oracle (allclose atol 2e-2, rtol 1e-2, as the
contiguous attention tests); a page id out of range sets device status 3
without faulting."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import attention as oa
from tests import _capi as C

pytestmark = pytest.mark.gpu

NAN_BF16 = np.uint16(0x7FC0)


def make_pages(k, v, page_size, seed, extra_pages=3):
    """Scatter contiguous k/v [B, Hkv, L, D] into shuffled pages; rows past L
    in the last page of each sequence (and the spare pages) hold NaN."""
    B, Hkv, L, D = k.shape
    per_seq = (L + page_size - 1) // page_size
    num_pages = B * per_seq + extra_pages
    rng = np.random.default_rng(seed)
    order = rng.permutation(num_pages)
    kp = np.full((num_pages, Hkv, page_size, D), NAN_BF16, dtype=np.uint16)
    vp = np.full((num_pages, Hkv, page_size, D), NAN_BF16, dtype=np.uint16)
    table = np.zeros((B, per_seq + 2), dtype=np.int32)
    for b in range(B):
        for j in range(per_seq):
            pg = order[b * per_seq + j]
            table[b, j] = pg
            rows = min(page_size, L - j * page_size)
            kp[pg, :, :rows] = k[b, :, j * page_size: j * page_size + rows]
            vp[pg, :, :rows] = v[b, :, j * page_size: j * page_size + rows]
        table[b, per_seq:] = -7  # past the sequence: never read
    return kp, vp, table


def dev_i32(a, device):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(device)


@pytest.mark.parametrize("page_size", [16, 32, 64, 128])
@pytest.mark.parametrize("B,L", [(1, 1000), (4, 4096), (2, 77)])
def test_full_length_pages_equal_contiguous_bits(cuda, page_size, B, L):
    q, k, v = oa.random_case(B, 32, 8, L, 128, seed=L + page_size)
    kp, vp, table = make_pages(k, v, page_size, seed=B)
    dq, dk, dv = (C.to_dev_bf16(a, cuda) for a in (q, k, v))
    want = C.attention(dq, dk, dv)
    got = C.paged_attention(dq, C.to_dev_bf16(kp, cuda), C.to_dev_bf16(vp, cuda), dev_i32(table, cuda),
                            dev_i32(np.full(B, L), cuda), L)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("page_size", [16, 128])
def test_variable_lengths_match_oracle(cuda, page_size):
    lens = np.array([1, 77, 512, 3000, 4096, 63], dtype=np.int32)
    B, max_len = len(lens), 4096
    q, k, v = oa.random_case(B, 32, 8, max_len, 128, seed=5 + page_size)
    kp, vp, table = make_pages(k, v, page_size, seed=9)
    ref = oa.decode_attention_paged(q, kp, vp, table, lens)
    got = C.paged_attention(C.to_dev_bf16(q, cuda), C.to_dev_bf16(kp, cuda), C.to_dev_bf16(vp, cuda),
                            dev_i32(table, cuda), dev_i32(lens, cuda), max_len)
    g = C.bf16_bits(got)
    from oracle.w4a16 import bf16_to_f32
    a, r = bf16_to_f32(g), bf16_to_f32(ref)
    assert np.all(np.isfinite(a))
    assert np.allclose(a, r, atol=2e-2, rtol=1e-2), np.abs(a - r).max()


def test_grouping_one_and_sixteen(cuda):
    for Hq, Hkv in ((8, 8), (32, 2)):
        lens = np.array([300, 1], dtype=np.int32)
        q, k, v = oa.random_case(2, Hq, Hkv, 512, 128, seed=Hq)
        kp, vp, table = make_pages(k, v, 32, seed=3)
        ref = oa.decode_attention_paged(q, kp, vp, table, lens)
        got = C.paged_attention(C.to_dev_bf16(q, cuda), C.to_dev_bf16(kp, cuda), C.to_dev_bf16(vp, cuda),
                                dev_i32(table, cuda), dev_i32(lens, cuda), 512)
        from oracle.w4a16 import bf16_to_f32
        assert np.allclose(bf16_to_f32(C.bf16_bits(got)), bf16_to_f32(ref), atol=2e-2, rtol=1e-2)


def test_bad_page_id_sets_status(cuda):
    from focal_b200 import _lib

    L = _lib.lib()
    q, k, v = oa.random_case(1, 32, 8, 256, 128, seed=1)
    kp, vp, table = make_pages(k, v, 64, seed=1)
    table[0, 1] = kp.shape[0]  # one past the last page
    assert L.focal_reset_device_status() == 0
    C.paged_attention(C.to_dev_bf16(q, cuda), C.to_dev_bf16(kp, cuda), C.to_dev_bf16(vp, cuda),
                      dev_i32(table, cuda), dev_i32(np.array([256]), cuda), 256)
    torch.cuda.synchronize()
    status = ctypes.c_int(-1)
    assert L.focal_device_status(status) == 0 and status.value == 3
    assert L.focal_reset_device_status() == 0


def test_torch_api_matches_capi(cuda):
    import focal_b200 as F

    lens = np.array([100, 2000], dtype=np.int32)
    q, k, v = oa.random_case(2, 32, 8, 2048, 128, seed=4)
    kp, vp, table = make_pages(k, v, 64, seed=4)
    args = (C.to_dev_bf16(q, cuda), C.to_dev_bf16(kp, cuda), C.to_dev_bf16(vp, cuda), dev_i32(table, cuda),
            dev_i32(lens, cuda))
    a = F.gqa_decode_attention_paged(*args, 2048)
    b = C.paged_attention(*args, 2048)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
