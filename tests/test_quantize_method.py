"""The int8 KV quantiser's division-free rounding, checked on the CPU.

The kernels (`quantize_s8` in doe_b200/csrc/common.cuh) compute
clamp(rint(x / s), -127, 127) for f16 values x and the f16 row scale s without
an IEEE division: y0 = x * rcp(s), y = fma(fma(-y0, s, x), rcp(s), y0), then
round-to-nearest-even (a clamp to +-127 in f32 and an add of 1.5 * 2^23,
whose low byte is the int8 value).  The CPU definition (oracle/doe_oracle.c, the int8
append) divides.  This test replays the kernels' arithmetic in float32 with an
exact-product FMA and requires the same integers as the division: every
positive and negative f16 value against a sample of f16 scales, exact
half-integer quotients and their f16 neighbours, and random rows with the
scale taken from the row maximum as the kernels take it.
"""
import numpy as np

F32, F64 = np.float32, np.float64


def _fma(a, b, c):
    # a * b is exact in float64 (24 + 24 bits); the sum rounds once in float64
    # and once to float32, which is exact here because the residual x - y0*s
    # is representable and the final correction is far below half an ulp.
    return (a.astype(F64) * b.astype(F64) + c.astype(F64)).astype(F32)


def kernel_quantize(x, s):
    rs = (F32(1.0) / s).astype(F32)  # correctly rounded reciprocal
    y0 = (x * rs).astype(F32)
    y = _fma(_fma(-y0, s, x), rs, y0)
    # clamp in f32, then round by adding 1.5 * 2^23 (round-half-even in f32)
    c = np.clip(y, F32(-127), F32(127)).astype(F32)
    bits = (c + F32(12582912.0)).astype(F32).view(np.uint32)
    return (bits & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)


def divide_quantize(x, s):
    return np.clip(np.rint((x / s).astype(F32)).astype(np.int64), -127, 127)


def _f16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(F32)


def test_every_f16_value_against_sampled_scales():
    g = np.random.default_rng(5)
    allx = _f16(np.arange(0, 0x7C00, dtype=np.uint16))
    allx = np.concatenate([allx, -allx])
    scales = [*_f16(g.integers(1, 0x7BFF, 24)), *_f16([0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF])]
    for s in scales:
        x = allx[np.abs(allx) <= F32(127.1) * s]  # |x| <= absmax = ~127 s
        if x.size:
            s_arr = np.full_like(x, s)
            np.testing.assert_array_equal(kernel_quantize(x, s_arr), divide_quantize(x, s_arr))


def test_exact_half_integer_quotients_and_neighbours():
    for sv in (0.0123, 1.0, 3.1e-5, 7.0e-8, 2.0 ** -20, 0.37):
        s = F32(np.float16(sv))
        if s == 0:
            continue
        base = ((np.arange(-128, 128).astype(F32) + F32(0.5)) * s).astype(np.float16)
        x = np.concatenate([base, np.nextafter(base, np.float16(np.inf)),
                            np.nextafter(base, np.float16(-np.inf))]).astype(F32)
        s_arr = np.full_like(x, s)
        np.testing.assert_array_equal(kernel_quantize(x, s_arr), divide_quantize(x, s_arr))


def test_random_rows_with_row_scales():
    g = np.random.default_rng(6)
    for _ in range(20):
        mag = 10.0 ** g.uniform(-9, 4)
        x = (g.standard_normal((512, 128)) * mag).astype(np.float16).astype(F32)
        s = (np.abs(x).max(axis=1, keepdims=True) / F32(127)).astype(F32).astype(np.float16).astype(F32)
        keep = (s != 0)[:, 0]
        x, s = x[keep], np.broadcast_to(s[keep], x[keep].shape)
        np.testing.assert_array_equal(kernel_quantize(x, s), divide_quantize(x, s))


def _rn32(fr):
    """Exact round-to-nearest-even of a rational to float32 (as a Fraction)."""
    from fractions import Fraction as Fr

    if fr == 0:
        return Fr(0)
    sign, a = (-1 if fr < 0 else 1), abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fr(2) ** e > a:
        e -= 1
    if Fr(2) ** (e + 1) <= a:
        e += 1
    sh = 149 if e < -126 else 23 - e
    m = a * Fr(2) ** sh
    n = m.numerator // m.denominator
    rem = m - n
    if rem > Fr(1, 2) or (rem == Fr(1, 2) and n % 2 == 1):
        n += 1
    return sign * Fr(n) / Fr(2) ** sh


def test_row_scale_quotient_is_correctly_rounded_for_every_f16():
    """div127 (common.cuh): q0 = amax * RN(1/127), q = fma(fma(-q0, 127, amax),
    RN(1/127), q0) equals RN_f32(amax / 127) for every finite f16 amax >= 0,
    each FMA modelled exactly (one rounding of the exact value)."""
    from fractions import Fraction as Fr

    r = _rn32(Fr(1, 127))
    assert float(r) == float.fromhex("0x1.020408p-7")
    for v in _f16(np.arange(0, 0x7C00, dtype=np.uint16)).astype(np.float64):
        a = Fr(float(v))
        q0 = _rn32(a * r)
        q = _rn32(_rn32(a - q0 * 127) * r + q0)
        assert q == _rn32(a / 127), v


def test_normal_scale_needs_no_clamp():
    """quantize_s8x2_normal skips the clamp when s = f16(amax / 127) is a normal
    f16: the row maximum itself (the largest quotient) must already land in
    [-127, 127], with and without the clamp, for every f16 amax."""
    amax = _f16(np.arange(1, 0x7C00, dtype=np.uint16))
    s = (amax.astype(np.float64) / 127).astype(F32).astype(np.float16).astype(F32)
    normal = (s >= F32(2.0 ** -14)) & (s <= F32(65504))
    x, s = amax[normal], s[normal]
    rs = (F32(1.0) / s).astype(F32)
    y0 = (x * rs).astype(F32)
    y = _fma(_fma(-y0, s, x), rs, y0)
    assert np.abs(y).max() < 127.5
    bits = (y + F32(12582912.0)).astype(F32).view(np.uint32)
    q = (bits & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
    np.testing.assert_array_equal(q, divide_quantize(x, s))
    np.testing.assert_array_equal(q, divide_quantize(-x, s) * -1)
