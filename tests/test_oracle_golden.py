"""Pin the numpy oracle to fixtures produced by the reference's own code.

The fixtures come from tests/golden/make_golden.py, which imports the
reference's focal_w4a16 package (pack_int4_weight, dequant_ref and the
bench/bench_w4a16.py:42-45 dequant-then-matmul).  CPU only.
"""
import numpy as np
import pytest

from oracle import w4a16 as ow


def load(golden_dir, name):
    return dict(np.load(golden_dir / name))


def test_pack_matches_reference(golden_dir):
    d = load(golden_dir, "pack.npz")
    assert np.array_equal(ow.pack_int4(d["q"]), d["packed"])
    assert np.array_equal(ow.pack_int4(d["ka_q"]), d["ka_packed"])
    # README.md:68-73 by hand: value k of the row at bits 4*(k%8) of word k//8
    assert d["ka_packed"].view(np.uint32)[0, 0] == 0x76543210
    assert d["ka_packed"].view(np.uint32)[0, 1] == 0x89ABCDEF
    assert d["ka_packed"].view(np.uint32)[1, 0] == 0xFFFFFFFF


def test_unpack_round_trips(golden_dir):
    d = load(golden_dir, "pack.npz")
    assert np.array_equal(ow.unpack_int4(d["packed"]), d["q"] & 0xF)


@pytest.mark.parametrize("name", ["baseline", "refstyle"])
def test_dequant_bit_exact(golden_dir, name):
    d = load(golden_dir, f"dequant_{name}.npz")
    got = ow.dequant(d["wq"], d["scales"], d["zeros"], int(d["K"]))
    assert got.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), d["deq"].view(np.uint32))


def test_dequant_products_are_exact_in_fp32(golden_dir):
    """(q - z) * s is exactly representable for both generators, so any fp32
    evaluation order (e.g. fma(q, s, -z*s)) reproduces dequant_ref bit-exactly."""
    for name in ("baseline", "refstyle"):
        d = load(golden_dir, f"dequant_{name}.npz")
        q = ow.unpack_int4(d["wq"]).astype(np.float64)
        s = np.repeat(d["scales"].astype(np.float64), 128, axis=1)
        z = np.repeat(d["zeros"].astype(np.float64), 128, axis=1)
        exact = (q - z) * s
        assert np.array_equal(exact.astype(np.float32).astype(np.float64), exact)
        fma_form = q * s - z * s
        assert np.array_equal(fma_form, exact)


@pytest.mark.parametrize("name", ["linear_k512_n128.npz", "linear_k1024_n192.npz"])
def test_linear_matches_reference(golden_dir, name):
    d = load(golden_dir, name)
    for M in (1, 2, 4, 8):
        y = ow.linear(d[f"x{M}"], d["wq"], d["scales"], d["zeros"])
        rep = ow.allclose_report(y, d[f"y{M}"])
        assert rep["allclose"], rep
        # fp32 summation order only: at most one bf16 rounding step apart
        diff = np.abs(ow.bf16_to_f32(y).astype(np.float64) - ow.bf16_to_f32(d[f"y{M}"]))
        ulp = np.abs(ow.bf16_to_f32(d[f"y{M}"]).astype(np.float64)) * 2.0**-7 + 1e-30
        assert np.all(diff <= ulp * 1.0001)


def test_linear_refstyle_generator(golden_dir):
    d = load(golden_dir, "linear_refstyle_m4.npz")
    y = ow.linear(d["x"], d["wq"], d["scales"], d["zeros"])
    assert ow.allclose_report(y, d["y"])["allclose"]


def test_structured_nibble_order(golden_dir):
    d = load(golden_dir, "structured.npz")
    M, K, N = int(d["M"]), int(d["K"]), int(d["N"])
    q_row = (np.arange(K) % 16).astype(np.uint8)
    assert np.array_equal(ow.pack_int4(q_row[None, :])[0], d["wq_row"])
    wq = np.repeat(d["wq_row"][None, :], 8, axis=0)  # every row of the fixture is identical
    s = np.full((8, K // 128), 0.01, np.float16)
    z = np.full((8, K // 128), 7.0, np.float16)
    y = ow.linear(d["x"], wq, s, z)
    for ref in (d["y_direct"][:, :8], d["y_packed"][:, :8]):
        assert ow.allclose_report(y, ref)["allclose"]


def test_bf16_round_trip_and_rounding():
    vals = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -2.5, 0.0, np.inf], np.float32)
    b = ow.f32_to_bf16(vals)
    # ties go to even: 1 + 2^-8 -> 1.0, 1 + 3*2^-8 -> 1 + 2^-6
    assert list(ow.bf16_to_f32(b)) == [1.0, 1.0, 1.0 + 2**-6, -2.5, 0.0, np.inf]


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (8, 4096, 11008), (4, 11008, 4096), (2, 8192, 8192)])
def test_threaded_cpu_baseline_matches_pinned_linear(M, K, N):
    """The timed CPU baseline (linear_threaded, which bench.py's cpu_baseline leg
    and --impl reference time) equals the fixture-pinned oracle linear to within
    one bf16 ulp per element: the same fp32 dequant and accumulation, only the
    BLAS blocking differs."""
    x, wq, s, z = ow.baseline_case(M, K, N, seed=77 + M)
    a = ow.bf16_to_f32(ow.linear_threaded(x, wq, s, z, threads=4)).astype(np.float64)
    b = ow.bf16_to_f32(ow.linear(x, wq, s, z)).astype(np.float64)
    ulp = np.abs(b) * 2.0 ** -7 + 1e-30  # one bf16 ulp (8 significant bits) at |b|
    assert np.all(np.abs(a - b) <= ulp), float(np.max(np.abs(a - b) / ulp))
