"""The row kernels encode FP8 codes from x / scale computed in five flops
(div_by_rcp in microserve_b200/csrc/common.cuh): r = RN(1/s), q0 = RN(x*r),
q1 = RN(q0 + r*RN(x - s*q0)), q2 = RN(q1 + r*RN(x - s*q1)), zeros passed through.
The reference divides (microserve/layers/fp8_linear.py:20-21, the oracle's
quantize_rows), so the codes are bit-exact only if q2 is the IEEE quotient.

This restates the sequence in exact rational arithmetic with binary32 rounding
after every operation (an FMA rounds once) and checks q2 == RN(x/s) on fp16
inputs and the scales the encoders produce (max(amax, 1e-8) * RN(1/448)), and
that the first remainder can be inexact (why one correction step is not used).
The CUDA code itself is held to the oracle's division in the GPU tests."""
import random
from fractions import Fraction as F

import numpy as np


def rn32(v: F) -> F:
    """Round a rational to the nearest binary32, ties to even (normal range)."""
    if v == 0:
        return F(0)
    sign = -1 if v < 0 else 1
    a = -v if v < 0 else v
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while F(2) ** e > a:
        e -= 1
    while F(2) ** (e + 1) <= a:
        e += 1
    assert e >= -126, "subnormal result"
    ulp = F(2) ** (e - 23)
    m = a / ulp
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return sign * fl * ulp


def fma(a: F, b: F, c: F) -> F:
    v = a * b + c
    return rn32(v) if v != 0 else F(0)


def div_by_rcp(x: F, s: F, r: F) -> F:
    q0 = rn32(x * r)
    q1 = fma(fma(-q0, s, x), r, q0)
    return fma(fma(-q1, s, x), r, q1)


def _cases(n: int, seed: int):
    rng = random.Random(seed)
    inv448 = rn32(F(1, 448))
    for _ in range(n):
        amax = float(np.float16(abs(rng.gauss(0, 1)) * 10 ** rng.uniform(-4, 4)))
        if amax == 0.0 or not np.isfinite(amax):
            continue
        s = rn32(F(max(amax, 1e-8)) * inv448)
        x = F(float(np.float16(rng.uniform(-1, 1) * amax)))
        if x != 0:
            yield x, s


def test_two_step_correction_is_the_ieee_quotient():
    n = 0
    for x, s in _cases(4000, seed=11):
        r = rn32(1 / s)
        assert div_by_rcp(x, s, r) == rn32(x / s), (float(x), float(s))
        n += 1
    assert n > 3500


def test_extremes_of_the_encoder_range():
    inv448 = rn32(F(1, 448))
    for amax in (float(np.float16(65504)), 1.0, float(np.float16(6e-8)), 3.0e-5):
        s = rn32(F(max(amax, 1e-8)) * inv448)
        r = rn32(1 / s)
        for x in (F(amax), F(-amax), F(float(np.float16(amax / 3))), F(float(np.float16(6e-8)))):
            if x != 0:
                assert div_by_rcp(x, s, r) == rn32(x / s), (float(x), float(s))


def test_first_remainder_can_be_inexact():
    """RN(x*r) is not always faithful, so the remainder after it is not always
    exact: the reason for the second correction."""
    inexact = 0
    for x, s in _cases(60000, seed=0):
        r = rn32(1 / s)
        q0 = rn32(x * r)
        rem = x - s * q0
        if rem != 0 and rn32(rem) != rem:
            inexact += 1
        if inexact:
            break
    assert inexact > 0
