"""The oracle's unit-tiled format (no GPU): it round-trips to the reference
packing bit for bit, and its bytes sit where the format says."""
import numpy as np
import pytest

from oracle import w4a16 as ow


@pytest.mark.parametrize("K,N", [(256, 64), (1024, 192), (11008, 128), (4096, 256)])
def test_tile_round_trip(K, N):
    _, wq, s, z = ow.baseline_case(1, K, N, seed=K + N)
    t = ow.tile_pack(wq, s, z, K)
    assert t.dtype == np.uint8 and t.size == (N // 64) * (K // 256) * ow.TILE_BYTES
    wq2, s2, z2 = ow.tile_unpack(t, K, N)
    assert np.array_equal(wq2, wq)
    assert np.array_equal(s2.view(np.uint16), s.view(np.uint16))
    assert np.array_equal(z2.view(np.uint16), z.view(np.uint16))


def test_tile_byte_positions():
    K, N = 1024, 192
    _, wq, s, z = ow.baseline_case(1, K, N, seed=11)
    t = ow.tile_pack(wq, s, z, K)
    TS = K // 256
    for rb in range(N // 64):
        for st in range(TS):
            base = (rb * TS + st) * ow.TILE_BYTES
            for r in (0, 7, 8, 63):
                row = 64 * rb + r
                for c in range(8):
                    pos = c ^ (r & 7)
                    got = t[base + 128 * r + 16 * pos: base + 128 * r + 16 * pos + 16].view(np.int32)
                    assert np.array_equal(got, wq[row, 32 * st + 4 * c: 32 * st + 4 * c + 4])
                sc = t[base + 8192 + 4 * r: base + 8196 + 4 * r].view(np.uint16)
                ze = t[base + 8448 + 4 * r: base + 8452 + 4 * r].view(np.uint16)
                assert np.array_equal(sc, s[row, 2 * st: 2 * st + 2].view(np.uint16))
                assert np.array_equal(ze, z[row, 2 * st: 2 * st + 2].view(np.uint16))
