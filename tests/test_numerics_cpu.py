"""Host check of a numerical identity the softmax kernel relies on.

The f32 row softmax divides every e by the same row sum s.  The kernel takes
the quotient as e * (1/s) in f64 rounded once to f32 (a multiply instead of a
division per element) and falls back to the IEEE division for results below
2^-125.  The claim: for f32 e and s with a normal f32 quotient, that equals
the IEEE f32 division e / s.  (A quotient of two 24-bit numbers that is not a
rounding midpoint is at least 2^-49 relative away from every midpoint, and a
normal one is never exactly a midpoint; the two f64 roundings stay within
2^-52.)

numpy's f64 arithmetic and its f64 -> f32 conversion are IEEE round-to-nearest
-even, as the GPU's __drcp_rn / __dmul_rn / cvt.rn.f32.f64 are, so the numpy
restatement is bit-for-bit the kernel's computation.  The IEEE f32 quotient is
the f64 quotient rounded once to f32 (exact because 53 >= 2 * 24 + 2; S. A.
Figueroa, "When is double rounding innocuous?", SIGNUM Newsletter 30(3), 1995).
"""
from __future__ import annotations

import numpy as np


def _check(e: np.ndarray, s: np.ndarray) -> int:
    e = e.astype(np.float32)
    s = s.astype(np.float32)
    want = (e.astype(np.float64) / s.astype(np.float64)).astype(np.float32)
    got = (e.astype(np.float64) * (1.0 / s.astype(np.float64))).astype(np.float32)
    normal = np.abs(got) >= np.float32(2.0**-125)
    bad = normal & (got.view(np.uint32) != want.view(np.uint32))
    assert not bad.any(), (e[bad][:5], s[bad][:5], got[bad][:5], want[bad][:5])
    return int(normal.sum())


def test_division_through_an_f64_reciprocal_equals_ieee_division_random():
    rng = np.random.default_rng(2024)
    n = 3_000_000
    # softmax operands: e in (0, 1], s in [1, 2^24]
    e = np.exp2(rng.uniform(-124.0, 0.0, n))
    s = np.exp2(rng.uniform(0.0, 24.0, n))
    assert _check(e, s) > 0.8 * n  # the rest fall below 2^-125 (IEEE division there)
    # the general f32 range
    e = np.exp2(rng.uniform(-100.0, 100.0, n)) * rng.choice([-1.0, 1.0], n)
    s = np.exp2(rng.uniform(-20.0, 20.0, n))
    assert _check(e, s) > 0.95 * n


def test_division_through_an_f64_reciprocal_equals_ieee_division_near_midpoints():
    """Numerators built so that e / s lands next to an f32 rounding midpoint:
    e = f32(m * s) for midpoints m, and its neighbours; plus divisors with
    all-ones mantissas and powers of two."""
    rng = np.random.default_rng(7)
    n = 1_000_000
    s = rng.integers(1 << 23, 1 << 24, n).astype(np.float64) * 2.0 ** rng.integers(-23, 1, n)
    mid = (2 * rng.integers(1 << 23, 1 << 24, n) + 1).astype(np.float64) * 2.0**-25
    e0 = (mid * s).astype(np.float32)
    for step in (-1, 0, 1):
        e = np.nextafter(e0, np.float32(np.inf) if step > 0 else np.float32(-np.inf)) if step else e0
        _check(e, s)
    ones = np.float32(2.0 - 2.0**-23) * np.exp2(np.arange(-10, 11)).astype(np.float32)
    pows = np.exp2(np.arange(-10, 25)).astype(np.float32)
    e = rng.uniform(0.0, 1.0, 200_000).astype(np.float32)
    for d in np.concatenate([ones, pows]):
        _check(e, np.full(e.shape, d, np.float32))
