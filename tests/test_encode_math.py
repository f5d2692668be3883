"""Exactness arguments of the device row encoder (row_encode.cuh), checked on the CPU with
exact rational arithmetic: each binary32 operation of the device formula is restated as the
exact result rounded once to binary32 (round to nearest, ties to even), as IEEE fmul / fma
define it, and compared with the IEEE quotient the reference computes
(quantize_reference, project2_quant/src/cpu_quant.cpp:97-170: scale = amax / max_finite)."""
from fractions import Fraction

import numpy as np

TWO = Fraction(2)


def rn32(v: Fraction) -> Fraction:
    """v rounded to the nearest binary32 value (ties to even); normal range only."""
    if v == 0:
        return Fraction(0)
    sign = -1 if v < 0 else 1
    a = abs(v)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if TWO ** e > a:
        e -= 1  # now 2^e <= a < 2^(e+1)
    assert -126 <= e <= 127, "outside the normal binary32 range"
    scaled = a / TWO ** (e - 23)  # in [2^23, 2^24)
    m = scaled.numerator // scaled.denominator
    rem = scaled - m
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and m % 2 == 1):
        m += 1
    return sign * m * TWO ** (e - 23)


def test_rn32_agrees_with_numpy_float32():
    rng = np.random.default_rng(0)
    for v in rng.standard_normal(2000) * 10.0 ** rng.integers(-30, 30, 2000):
        assert rn32(Fraction(float(v))) == Fraction(float(np.float32(v)))


def test_fp8_scale_without_division_is_the_ieee_quotient():
    """scale = RN(amax / max_finite) as q0 = RN(amax * y), r = RN(amax - q0 * max_finite),
    RN(q0 + r * y) with y = RN(1 / max_finite), for every positive finite binary16 amax and
    both FP8 maxima (E4M3 448, E5M2 57344)."""
    halves = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    for max_finite, y_hex in ((448.0, "0x1.24924ap-9"), (57344.0, "0x1.24924ap-16")):
        b = Fraction(max_finite)
        y = Fraction(float.fromhex(y_hex))
        assert y == rn32(1 / b)
        for a_f in halves:
            a = Fraction(float(a_f))
            q0 = rn32(a * y)
            r = rn32(a - q0 * b)
            assert r == a - q0 * b, "the FMA residual is exact"
            assert rn32(q0 + r * y) == rn32(a / b), (max_finite, float(a_f))
