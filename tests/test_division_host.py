"""The fp32 division-by-constant scheme of the catalog kernels, restated in exact arithmetic.

The kernels divide an fp32 term by its per-launch divisor d with y = RN(1/d) and two quotient
corrections (P. Markstein, IBM J. Res. Dev. 34(1), 1990):

    q0 = RN(x*y); r0 = RN(x - q0*d); q1 = RN(q0 + r0*y); r1 = RN(x - q1*d); q = RN(q1 + r1*y)

(every RN one fp32 rounding, as an fma rounds), for |x| and |d| in [2^-60, 2^60]; everything
else takes IEEE division.  Here each step is computed exactly with fractions and rounded to
the nearest fp32 (ties to even), and q must equal the correctly rounded x/d — the quotient
numpy's fp32 division and eager torch give — for random operands across the exponent range and
for quotients close to rounding ties.
"""
from fractions import Fraction

import numpy as np
import pytest


def rn32(v: Fraction) -> Fraction:
    """v rounded to the nearest fp32 (ties to even); normal range only."""
    if v == 0:
        return Fraction(0)
    sign = -1 if v < 0 else 1
    a = abs(v)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    assert -126 <= e <= 127, "outside the normal range"
    scaled = a / Fraction(2) ** (e - 23)  # in [2^23, 2^24)
    m = scaled.numerator // scaled.denominator
    rem = scaled - m
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and m % 2 == 1):
        m += 1
    return sign * m * Fraction(2) ** (e - 23)


def div_by(x: Fraction, d: Fraction) -> Fraction:
    y = rn32(1 / d)
    q0 = rn32(x * y)
    r0 = rn32(x - q0 * d)
    q1 = rn32(q0 + r0 * y)
    r1 = rn32(x - q1 * d)
    return rn32(q1 + r1 * y)


def _f32(v) -> Fraction:
    return Fraction(float(np.float32(v)))


def _check(xs, ds):
    for x, d in zip(xs, ds):
        xf, df = _f32(x), _f32(d)
        want = Fraction(float(np.float32(x) / np.float32(d)))  # IEEE fp32 division
        assert div_by(xf, df) == want, (float(xf), float(df))


def test_random_operands_across_the_exponent_range():
    rng = np.random.default_rng(11)
    n = 4000
    xs = (rng.uniform(1, 2, n) * 2.0 ** rng.integers(-60, 60, n) * rng.choice([-1, 1], n)).astype(np.float32)
    ds = (rng.uniform(1, 2, n) * 2.0 ** rng.integers(-60, 60, n) * rng.choice([-1, 1], n)).astype(np.float32)
    _check(xs, ds)


@pytest.mark.parametrize("d", [3.0, 7.0, 0.1, 1 / 3, 1.5, 65537.0, -3.0, 1e-18, 1e18])
def test_quotients_next_to_rounding_ties(d):
    """x = d * (a tie point between two fp32 numbers), rounded to fp32: the quotient lands
    within a few ulps of x's precision of the tie, the hardest case for a corrected quotient."""
    rng = np.random.default_rng(int(abs(d) * 1000) % 2**32)
    df = _f32(d)
    xs = []
    for _ in range(400):
        m = int(rng.integers(2**23, 2**24))
        e = int(rng.integers(-20, 20))
        tie = (Fraction(2 * m + 1, 2)) * Fraction(2) ** (e - 23)
        xs.append(float(rn32(tie * df)))
    _check(xs, [d] * len(xs))


def test_small_integer_multiples_of_three():
    """Sums of three N(0,1) fp32 values divided by 3 (the 1-D mean): every exact multiple of
    three among small integers, and their neighbours."""
    xs = []
    for k in range(1, 3000):
        v = np.float32(k)
        xs += [v, np.nextafter(v, np.float32(0)), np.nextafter(v, np.float32(1e9))]
    _check(xs, [3.0] * len(xs))
