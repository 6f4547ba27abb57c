"""Unit-tiled weights on the GPU, through the C ABI: the device packer
matches the oracle byte for byte and its inverse restores the reference
packing bit for bit; the tiled linears give the same bits as the linears on
the reference layout (same arithmetic, same order)."""
import numpy as np
import pytest
import torch

from oracle import w4a16 as ow
from tests import _capi as C

pytestmark = pytest.mark.gpu

SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (8192, 8192), (1024, 192), (8192, 28672)]


@pytest.mark.parametrize("K,N", [(256, 64), (1024, 192), (11008, 4096), (4096, 11008)])
def test_device_pack_matches_oracle_and_round_trips(cuda, K, N):
    _, wq, s, z = ow.baseline_case(1, K, N, seed=K + 3 * N)
    dwq, ds, dz = (C.to_dev(a, cuda) for a in (wq, s, z))
    t = C.tile_pack(dwq, ds, dz)
    assert np.array_equal(t.cpu().numpy(), ow.tile_pack(wq, s, z, K))
    wq2, s2, z2 = C.tile_unpack(t, K, N)
    assert torch.equal(wq2, dwq) and torch.equal(s2.view(torch.int16), ds.view(torch.int16))
    assert torch.equal(z2.view(torch.int16), dz.view(torch.int16))


@pytest.mark.parametrize("K,N", SHAPES)
def test_tiled_linear_equals_reference_layout_linear(cuda, K, N):
    x8, wq, s, z = ow.baseline_case(8, K, N, seed=77 + K + N)
    dwq, ds, dz = (C.to_dev(a, cuda) for a in (wq, s, z))
    t = C.tile_pack(dwq, ds, dz)
    for M in (1, 2, 3, 4, 8):
        x = C.to_dev_bf16(x8[:M], cuda)
        a = C.gemv(x, dwq, ds, dz)
        b = C.gemv_tiled(x, t, N)
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), (M, K, N)
    fa = C.gemv(x, dwq, ds, dz, out_dtype=torch.float32)
    fb = C.gemv_tiled(x, t, N, out_dtype=torch.float32)
    assert torch.equal(fa.view(torch.int32), fb.view(torch.int32))
    if K * N <= 8192 * 8192:
        rep = ow.allclose_report(C.bf16_bits(b), ow.linear(x8, wq, s, z), 2e-2, 1e-2)
        assert rep["allclose"], rep


@pytest.mark.parametrize("M,K,N", [(1, 4096, 11008), (8, 4096, 11008), (4, 1024, 256)])
def test_tiled_gate_up_silu_equals_reference_layout(cuda, M, K, N):
    x, wg, sg, zg = ow.baseline_case(M, K, N, seed=900 + M)
    _, wu, su, zu = ow.baseline_case(1, K, N, seed=950 + M)
    dx = C.to_dev_bf16(x, cuda)
    gate = tuple(C.to_dev(a, cuda) for a in (wg, sg, zg))
    up = tuple(C.to_dev(a, cuda) for a in (wu, su, zu))
    a = C.gate_up_silu(dx, gate, up)
    b = C.gate_up_silu_tiled(dx, C.tile_pack(*gate), C.tile_pack(*up), N)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_torch_api_tiled_linear(cuda):
    import focal_b200 as F

    x, wq, s, z = F.baseline_case(4, 8192, 4096, seed=21, device=cuda)
    t = F.w4a16_tile_pack(wq, s, z)
    assert t.dtype == torch.uint8 and t.numel() == 4096 // 64 * (8192 // 256) * 8704
    a = F.w4a16_linear(x, wq, s, z)
    assert torch.equal(F.w4a16_linear_tiled(x, t, 4096).view(torch.int16), a.view(torch.int16))
    assert torch.equal(F.w4a16_linear_tiled_f32(x, t, 4096), F.w4a16_linear_f32(x, wq, s, z))
    with pytest.raises(RuntimeError, match="tiles must hold"):
        F.w4a16_linear_tiled(x, t[:-16], 4096)
