"""The decode kernel's 22-bit activation digits (csrc/tl_decode.cu: put_digits and
the gate/up epilogue's published act digits), restated in numpy.

X = rint(x 2^k), |X| <= 2^22, is split into balanced base-256 digits
X = 65536 d0 + 256 d1 + d2 with d1, d2 in [-128, 127].  The kernel gets X
from one fma with 1.5 * 2^23 (the float's bit pattern is 0x4B400000 + X) and
the digits as bytes of shifted copies of that pattern.  This checks, over
every X in range, that those bytes are the balanced digits, and that the fma
rounds like rint (round half to even).
"""
import numpy as np


def digits_reference(x):
    y = (x + 128) >> 8
    z = (y + 128) >> 8
    return z & 0xFF, y & 0xFF, x & 0xFF


def digits_from_bits(bits):
    d0 = ((bits + 32896 - 0x400000) & 0xFFFFFFFF) >> 16 & 0xFF
    d1 = ((bits + 128) >> 8) & 0xFF
    d2 = bits & 0xFF
    return d0, d1, d2


def s8(a):
    return np.where(a > 127, a - 256, a)


def test_bytes_are_the_balanced_digits_for_every_x():
    x = np.arange(-(1 << 22), (1 << 22) + 1, dtype=np.int64)
    bits = (0x4B400000 + x) & 0xFFFFFFFF
    ref = digits_reference(x)
    got = digits_from_bits(bits)
    for r, g in zip(ref, got):
        assert np.array_equal(r, g)
    d0, d1, d2 = (s8(v) for v in got)
    assert np.array_equal(65536 * d0 + 256 * d1 + d2, x)
    assert d1.min() >= -128 and d1.max() <= 127 and d2.min() >= -128 and d2.max() <= 127
    assert np.abs(d0).max() <= 64


def test_magic_fma_rounds_like_rint():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(1 << 20).astype(np.float32)
    for k in (0, 10, 20):
        p = v.astype(np.float64) * 2.0 ** k          # exact: a power-of-two scale
        p = p[np.abs(p) <= 2 ** 22]
        # fmaf(v, 2^k, 1.5 * 2^23): the exact sum, rounded once to float32
        s = (p + 12582912.0).astype(np.float32)
        got = s.view(np.uint32).astype(np.int64) - 0x4B400000
        assert np.array_equal(got, np.rint(p).astype(np.int64))
    # ties go to even, as __float2int_rn
    ties = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5], dtype=np.float64)
    s = (ties + 12582912.0).astype(np.float32)
    assert (s.view(np.uint32).astype(np.int64) - 0x4B400000).tolist() == [0, 2, 2, 0, -2, -2]
