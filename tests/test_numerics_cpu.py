"""Host check of a numerical identity the row kernels rely on.

The f32 row kernels divide every element of a row by the same value s (the
softmax's row sum, LayerNorm's sqrt(var + eps)).  Instead of an IEEE division
per element they take, once per row, the reciprocal as a pair
yh = RN(1/s), yl = RN(1/s - yh), and per element

    q0  = fma(e, yh, RN(e * yl))     within one ulp of e/s
    rem = fma(-q0, s, e)             exact (q0 is within one ulp)
    q   = fma(rem, yh, q0)           = RN(e / s)

(the correction step of P. Markstein, "Computation of elementary functions on
the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), falling
back to the IEEE division for results below 2^-125.  This test evaluates the
same f32 operations with exact rational arithmetic, rounding each to f32 (ties
to even) as the GPU's __fmaf_rn / __fmul_rn / __frcp_rn do, and checks the
result against the correctly rounded quotient: random operands, quotients
built next to rounding midpoints, and divisors with all-ones significands or
powers of two.
"""
from __future__ import annotations

import random
from fractions import Fraction as F

import numpy as np


def _rn32(x: F) -> float:
    """x rounded to the nearest f32, ties to even (normal range)."""
    if x == 0:
        return 0.0
    c = np.float32(float(x))
    cands = [np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))]
    return float(min(cands, key=lambda t: (abs(F(float(t)) - x), int(np.float32(t).view(np.uint32)) & 1)))


def _kernel_quotient(e: float, s: float) -> tuple[float, bool]:
    yh = _rn32(F(1) / F(s))
    yl = _rn32(F(1) / F(s) - F(yh))
    q0 = _rn32(F(e) * F(yh) + F(_rn32(F(e) * F(yl))))
    rem = F(e) - F(q0) * F(s)
    exact = F(_rn32(rem)) == rem
    return _rn32(F(q0) + F(_rn32(rem)) * F(yh)), exact


def _check(e: float, s: float) -> bool:
    e = float(np.float32(e))
    s = float(np.float32(s))
    want = _rn32(F(e) / F(s))
    if e == 0 or abs(want) < 2.0**-125:
        return False  # the kernel takes the IEEE division there
    got, exact = _kernel_quotient(e, s)
    assert exact, ("remainder not exact", e, s)
    assert got == want, (e, s, got, want)
    return True


def test_row_division_equals_ieee_division_random():
    rng = random.Random(2024)
    # softmax: e in (0, 1], s in [1, 2^24]
    checked = sum(_check(2.0 ** rng.uniform(-100.0, 0.0), 2.0 ** rng.uniform(0.0, 24.0)) for _ in range(8000))
    assert checked > 6000
    # LayerNorm: (x - mean) of either sign over denom = sqrt(var + eps)
    checked = sum(_check(rng.choice([-1.0, 1.0]) * 2.0 ** rng.uniform(-60.0, 60.0), 2.0 ** rng.uniform(-30.0, 30.0))
                  for _ in range(8000))
    assert checked > 6000


def test_row_division_equals_ieee_division_near_midpoints():
    rng = random.Random(7)
    for _ in range(5000):
        s = rng.randint(1 << 23, (1 << 24) - 1) * 2.0 ** rng.randint(-23, 0)
        mid = (2 * rng.randint(1 << 23, (1 << 24) - 1) + 1) * 2.0**-25
        e0 = np.float32(mid * s)
        for e in (np.nextafter(e0, np.float32(-1)), e0, np.nextafter(e0, np.float32(2))):
            _check(float(e), s)
    for k in range(-4, 5):
        for d in ((2.0 - 2.0**-23) * 2.0**k, 2.0**k, 3.0 * 2.0**k):
            for _ in range(300):
                _check(rng.uniform(0.0, 1.0), d)
