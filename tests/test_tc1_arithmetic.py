"""The exactness claims of the tensor-core batch-1 kernel, checked on the
host (no GPU).  gemv_tc1 (flatrun_b200/csrc/gemv_tc1.cuh) computes the
reference's fp32 dot products with fp16 tensor-core operands; this file
restates how it forms those operands, bit for bit, in NumPy and checks
exhaustively that no operand is rounded:

* weights (tc1_sb): a quant value q of a sub-block with 6-bit scale sc enters
  the MMA as the fp16 FMA (1024 + q) * sc - 1024 * sc (low nibbles; the
  nibble or'ed into the mantissa of 1024, bits 0x6400) or
  (1024 + 16 q) * (sc / 16) - 64 * sc (high nibbles, in place), rounded once;
  the scale pairs are themselves formed by fp16 arithmetic from 1024 + sc.
  For every q < 16 (Q4_K) and q < 32 (Q5_K, the fifth bit joined below the
  bias) and every sc < 64 the result is exactly q * sc;
* activations (tc1_scale, split3): each super-block of x is scaled by a power
  of two s with |x s| < 2^15 and written as hi + mid + lo, three
  round-to-nearest fp16 terms formed in fp32; their sum is x s exactly for
  every element down to 2^-9 of the super-block's largest, and short of it
  by less than 2^-24 (half an fp16 subnormal step, in scaled units) below;
* products: an fp16 x fp16 product has at most 22 significant bits, so the
  MMA's products are exact in its fp32 accumulator."""

from __future__ import annotations

import numpy as np

F16 = np.float16


def f16_bits(v: int) -> np.float16:
    return np.array([v], dtype=np.uint16).view(np.float16)[0]


def fma16(a, b, c) -> np.float16:
    """fp16 fused multiply-add: exact in float64 (operands have 11 bits), one
    rounding to fp16 (round to nearest even)."""
    return F16(float(a) * float(b) + float(c))


def test_scale_pairs_are_exact():
    bias = f16_bits(0x6400)  # 1024
    for sc in range(64):
        with_sc = f16_bits(0x6400 | sc)  # prmt(sc, bias): 1024 + sc
        assert float(with_sc) == 1024 + sc
        sl = F16(float(with_sc) + float(F16(-1024.0)))  # hadd2(.., -1024)
        assert float(sl) == sc
        assert float(F16(float(sl) * -1024.0)) == -1024 * sc  # hmul2(sl, -1024)
        sg = fma16(with_sc, F16(1 / 16), F16(-64.0))  # hfma2(.., 1/16, -64)
        assert float(sg) == sc / 16
        assert float(F16(float(sg) * -1024.0)) == -64 * sc
    assert float(bias) == 1024.0


def test_weight_operands_are_exact_q_times_sc():
    for sc in range(64):
        s_lo, n_lo = F16(sc), F16(-1024 * sc)
        s_hi, n_hi = F16(sc / 16), F16(-64 * sc)
        for q in range(32):  # Q4_K: q < 16; Q5_K: q < 32 with the fifth bit
            lo = f16_bits(0x6400 | q)  # bit 4 of a low lane is Q5_K's fifth bit
            assert float(lo) == 1024 + q
            assert float(fma16(lo, s_lo, n_lo)) == q * sc
            hi = f16_bits(0x6400 | (q << 4))  # high nibble in place, fifth bit at bit 8
            assert float(hi) == 1024 + 16 * q
            assert float(fma16(hi, s_hi, n_hi)) == q * sc


def split3(xs: np.ndarray):
    """split3 of gemv_tc1.cuh: round-to-nearest fp16 terms formed in fp32."""
    xs = xs.astype(np.float32)
    h0 = xs.astype(np.float16)
    r = (xs - h0.astype(np.float32)).astype(np.float32)
    h1 = r.astype(np.float16)
    h2 = (r - h1.astype(np.float32)).astype(np.float32).astype(np.float16)
    return h0, h1, h2


def scale_of(m: float):
    """tc1_scale: s = 2^(14 - floor(log2 m)), exponent clamped to [-113, 100]."""
    e = int((np.float32(m).view(np.uint32) >> 23) & 0xFF) - 127
    se = min(100, max(-113, 14 - e))
    return np.float32(2.0 ** se), np.float32(2.0 ** -se)


def test_activation_terms_sum_to_x_exactly():
    rng = np.random.default_rng(5)
    for trial in range(400):
        decades = rng.uniform(0, 60)
        x = (rng.standard_normal(256) * 10.0 ** rng.uniform(-decades / 2, decades / 2, 256)).astype(np.float32)
        x *= np.float32(10.0 ** rng.uniform(-20, 20))
        x = np.where(np.isfinite(x), x, np.float32(0.0)).astype(np.float32)
        if trial % 7 == 0:
            x[rng.integers(0, 256, 16)] = 0.0
        m = float(np.abs(x).max())
        if m == 0.0 or not np.isfinite(m):
            continue
        s, inv = scale_of(m)
        assert s * inv == 1.0
        xs = (x * s).astype(np.float32)
        # a power of two: exact wherever x s is a normal fp32 number (elements
        # below 2^-126 in scaled units, 2^-140 of the largest, may lose bits)
        normal = np.abs(xs) >= 2.0 ** -126
        assert np.all(xs[normal].astype(np.float64) == x[normal].astype(np.float64) * float(s))
        if m >= 2.0 ** -86:
            assert 2.0 ** 14 <= np.abs(xs).max() < 2.0 ** 15
        else:  # the scale stays 2^100
            assert np.abs(xs).max() < 2.0 ** 14
        h0, h1, h2 = split3(xs)
        total = h0.astype(np.float64) + h1.astype(np.float64) + h2.astype(np.float64)
        err = np.abs(total - xs.astype(np.float64))
        big = np.abs(xs) >= 2.0 ** 14 * 2.0 ** -9
        assert np.all(err[big] == 0.0), trial
        assert np.all(err <= 2.0 ** -25), trial


def test_scale_covers_every_finite_fp32_maximum():
    """The largest finite fp32 values (up to 3.4e38) still scale below 2^15,
    so no fp16 term overflows; the smallest normal ones keep 1 / s normal."""
    for m in [np.finfo(np.float32).max, 2.0 ** 127, 2.0 ** 116, 5.06e34, 1.0, 2.0 ** -86, 2.0 ** -126]:
        s, inv = scale_of(float(m))
        assert np.isfinite(s) and np.isfinite(inv) and s * inv == 1.0
        assert float(np.float32(m)) * float(s) < 2.0 ** 15
        assert float(inv) >= 2.0 ** -126 and float(s) >= 2.0 ** -126


def test_fp16_products_fit_fp32():
    rng = np.random.default_rng(6)
    a = rng.standard_normal(100000).astype(np.float16)
    b = (rng.standard_normal(100000) * 100).astype(np.float16)
    exact = a.astype(np.float64) * b.astype(np.float64)
    assert np.all(exact.astype(np.float32).astype(np.float64) == exact)
