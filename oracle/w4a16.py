"""numpy restatement of the reference W4A16 algorithm — TEST INFRASTRUCTURE ONLY.

Parity PINNED: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by the reference's own Python module
(``tests/golden/make_golden.py``), bit-exactly for packing and dequant.

Reference semantics restated (paths relative to the reference project):

* packing, focal_w4a16/__init__.py:38-54 and README.md:66-73 — eight unsigned
  int4 values per int32 word, value ``k`` of a row stored at bits
  ``4*(k % 8) .. 4*(k % 8) + 3`` of word ``k // 8``.
* dequant, focal_w4a16/__init__.py:57-91 — ``w = (float(q) - float(z)) *
  float(s)`` in fp32, with ``s``/``z`` of the 128-wide K group ``k // 128``.
* linear, bench/bench_w4a16.py:42-45 and tests/test_correctness.py:55-56 —
  ``(x.float() @ w_deq.T).to(bfloat16)`` with fp32 accumulation.

bf16 values are carried as numpy ``uint16`` bit patterns; fp16 as
``float16``.  ``bf16_to_f32`` / ``f32_to_bf16`` implement the IEEE
round-to-nearest-even conversion that torch uses for ``.to(bfloat16)``.
"""
from __future__ import annotations

import numpy as np

GROUP = 128


# ----------------------------------------------------------------- bf16 bits
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bits, round-to-nearest-even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


# ------------------------------------------------------------------- packing
def pack_int4(q: np.ndarray) -> np.ndarray:
    """uint8 [N, K] (values 0..15 used, upper bits ignored) -> int32 [N, K/8].

    Follows focal_w4a16/__init__.py:50-53: ``packed |= (q[:, :, i] & 0xF) << 4i``.
    """
    q = np.asarray(q)
    if q.ndim != 2 or q.shape[1] % 8 != 0:
        raise ValueError("q must have shape [N, K] with K divisible by 8")
    n, k = q.shape
    q8 = (q.astype(np.uint32) & 0xF).reshape(n, k // 8, 8)
    packed = np.zeros((n, k // 8), dtype=np.uint32)
    for i in range(8):
        packed |= q8[:, :, i] << np.uint32(4 * i)
    return packed.view(np.int32)


def unpack_int4(wq: np.ndarray) -> np.ndarray:
    """int32 [N, K/8] -> uint8 [N, K]; focal_w4a16/__init__.py:85-88.

    Byte j of a little-endian word holds values 2j (low nibble) and 2j+1
    (high nibble), which is the reference's ``(word >> 4i) & 0xF`` order.
    """
    b = np.ascontiguousarray(wq, dtype=np.int32).view(np.uint8)
    n, nb = b.shape
    q = np.empty((n, nb, 2), dtype=np.uint8)
    np.bitwise_and(b, 0xF, out=q[:, :, 0])
    np.right_shift(b, 4, out=q[:, :, 1])
    return q.reshape(n, nb * 2)


# ------------------------------------------------------------------- dequant
def dequant(wq: np.ndarray, scales: np.ndarray, zeros: np.ndarray, K: int) -> np.ndarray:
    """fp32 [N, K] = (q - z) * s, exactly as focal_w4a16/__init__.py:86-91.

    Every step is an fp32 operation with the same operand order as the
    reference (q and z widened to fp32, one subtraction, one multiplication),
    so the result is bit-identical.
    """
    if K % GROUP != 0:
        raise ValueError("K must be divisible by 128")
    wq = np.asarray(wq, dtype=np.int32)
    n, kw = wq.shape
    if kw * 8 != K:
        raise ValueError("wq shape does not match K")
    scales = np.asarray(scales, dtype=np.float16)
    zeros = np.asarray(zeros, dtype=np.float16)
    if scales.shape != (n, K // GROUP) or zeros.shape != (n, K // GROUP):
        raise ValueError("scales/zeros must have shape [N, K / 128]")
    w = unpack_int4(wq).astype(np.float32).reshape(n, K // GROUP, GROUP)
    np.subtract(w, zeros.astype(np.float32)[:, :, None], out=w)   # q - z   (fp32)
    np.multiply(w, scales.astype(np.float32)[:, :, None], out=w)  # * s     (fp32)
    return w.reshape(n, K)


# -------------------------------------------------------------------- linear
def linear(x_bf16: np.ndarray, wq: np.ndarray, scales: np.ndarray, zeros: np.ndarray,
           out: str = "bf16") -> np.ndarray:
    """The reference's ``baseline_dequant_matmul`` (bench/bench_w4a16.py:42-45).

    ``x_bf16`` is uint16 bf16 bits [M, K].  The product is accumulated in fp32
    (numpy sgemm), then rounded to bf16 bits (``out="bf16"``) or returned as
    fp32 (``out="f32"``, the row-parallel partial-sum form).
    """
    x = bf16_to_f32(x_bf16)
    K = x.shape[1]
    w = dequant(wq, scales, zeros, K)
    y = x @ w.T
    if out == "f32":
        return y.astype(np.float32)
    return f32_to_bf16(y)


def linear_f64(x_bf16: np.ndarray, wq: np.ndarray, scales: np.ndarray,
               zeros: np.ndarray) -> np.ndarray:
    """Same product accumulated in float64 (no rounding) — the exact value the
    fp32 paths approximate; used to bound accumulation-order error."""
    x = bf16_to_f32(x_bf16).astype(np.float64)
    K = x.shape[1]
    w = dequant(wq, scales, zeros, K).astype(np.float64)
    return x @ w.T


# -------------------------------------------------------- unit-tiled format
# Not a reference format: the re-layout the reference lists as next work
# (docs/blog_notes.md:193-213), restated here so the device packer can be
# checked byte for byte; its inverse must give back the reference packing.
TILE_BYTES = 8704


def tile_pack(wq: np.ndarray, scales: np.ndarray, zeros: np.ndarray, K: int) -> np.ndarray:
    """(wq [N, K/8] int32, scales / zeros [N, K/128] fp16) -> uint8 tiles.

    Unit u = rb * (K/256) + st, 8704 bytes: 64 rows x 32 words with row r at
    byte 128 r and its 16-byte chunk c at position c ^ (r & 7); then the rows'
    scale pairs (groups 2 st, 2 st + 1, 4 bytes a row), then their zero pairs.
    """
    N = wq.shape[0]
    RB, TS = N // 64, K // 256
    w = np.ascontiguousarray(wq).view(np.uint32).reshape(RB, 64, TS, 8, 4)   # [rb, r, st, c, word]
    w = w.transpose(0, 2, 1, 3, 4)                                          # [rb, st, r, c, word]
    r = np.arange(64)[:, None]
    pos = np.arange(8)[None, :]
    c_at_pos = pos ^ (r & 7)                                                # chunk stored at position
    w = np.take_along_axis(w, np.broadcast_to(c_at_pos[None, None, :, :, None], w.shape), axis=3)
    sz = [np.ascontiguousarray(a).view(np.uint32).reshape(RB, 64, TS).transpose(0, 2, 1)
          for a in (scales, zeros)]                                         # [rb, st, r]
    out = np.empty((RB, TS, TILE_BYTES // 4), dtype=np.uint32)
    out[:, :, :2048] = w.reshape(RB, TS, 2048)
    out[:, :, 2048:2112] = sz[0]
    out[:, :, 2112:2176] = sz[1]
    return out.reshape(-1).view(np.uint8)


def tile_unpack(tiles: np.ndarray, K: int, N: int):
    """Inverse of tile_pack: (wq int32 [N, K/8], scales fp16, zeros fp16)."""
    RB, TS = N // 64, K // 256
    t = np.ascontiguousarray(tiles).view(np.uint32).reshape(RB, TS, TILE_BYTES // 4)
    w = t[:, :, :2048].reshape(RB, TS, 64, 8, 4)
    r = np.arange(64)[:, None]
    c = np.arange(8)[None, :]
    pos_of_c = c ^ (r & 7)                                                  # position holding chunk c
    w = np.take_along_axis(w, np.broadcast_to(pos_of_c[None, None, :, :, None], w.shape), axis=3)
    wq = w.transpose(0, 2, 1, 3, 4).reshape(N, K // 8).view(np.int32)
    sc = t[:, :, 2048:2112].transpose(0, 2, 1).reshape(N, K // 256).copy().view(np.float16)
    ze = t[:, :, 2112:2176].transpose(0, 2, 1).reshape(N, K // 256).copy().view(np.float16)
    return np.ascontiguousarray(wq), sc, ze


# ---------------------------------------------------------------- generators
def baseline_case(M: int, K: int, N: int, seed: int):
    """Inputs with the benchmark's value distributions, drawn by numpy.

    x ~ N(0,1) rounded to bf16; wq uniform random 32-bit words; scales fp16
    U[0.005, 0.02]; zeros fp16 integers U{0..15}.  (The product's own
    generator, ``focal_b200.baseline_case``, draws the same distributions on
    a seeded torch CPU generator.)
    """
    rng = np.random.default_rng(seed)
    x = f32_to_bf16(rng.standard_normal((M, K), dtype=np.float32))
    wq = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    scales = rng.uniform(0.005, 0.02, size=(N, K // GROUP)).astype(np.float16)
    zeros = rng.integers(0, 16, size=(N, K // GROUP)).astype(np.float16)
    return x, wq, scales, zeros


def allclose_report(y_bf16: np.ndarray, ref_bf16: np.ndarray, atol: float = 2e-2,
                    rtol: float = 1e-2) -> dict:
    """Both tolerance forms: allclose (|d| <= atol + rtol|ref|) and the
    reference's own max-abs / max-rel metric (tests/test_correctness.py:15-19)."""
    y = bf16_to_f32(y_bf16).astype(np.float64)
    r = bf16_to_f32(ref_bf16).astype(np.float64)
    d = np.abs(y - r)
    return {
        "allclose": bool(np.all(d <= atol + rtol * np.abs(r))),
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_rel": float((d / np.maximum(np.abs(r), 1.0)).max()) if d.size else 0.0,
    }


# ------------------------------------------------------- timed CPU baseline
def linear_threaded(x_bf16: np.ndarray, wq: np.ndarray, scales: np.ndarray, zeros: np.ndarray,
                    threads: int) -> np.ndarray:
    """``linear`` with the N rows split over ``threads`` worker threads.

    Each worker dequantises its row block (``dequant``) and multiplies it with
    single-threaded BLAS; numpy releases the GIL in both, so the blocks run in
    parallel.  Same arithmetic per element as ``linear`` (fp32 dequant, fp32
    accumulation, bf16 rounding).  Used as the timed CPU restatement of the
    reference's baseline_dequant_matmul.
    """
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    x = bf16_to_f32(x_bf16)
    K = x.shape[1]
    N = wq.shape[0]
    y = np.empty((x.shape[0], N), dtype=np.float32)
    rows = 256  # row blocks small enough that each block's temporaries stay in cache
    starts = range(0, N, rows)

    def work(a):
        b = min(N, a + rows)
        w = dequant(wq[a:b], scales[a:b], zeros[a:b], K)
        y[:, a:b] = x @ w.T

    with threadpool_limits(limits=1, user_api="blas"):
        with ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
            list(ex.map(work, starts))
    return f32_to_bf16(y)
