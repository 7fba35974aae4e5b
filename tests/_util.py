"""Helpers shared by the tests: ULP distance, bit-level comparison."""
from __future__ import annotations

import numpy as np


def ordered_bits(a: np.ndarray) -> np.ndarray:
    """Maps floats onto integers that order like the floats (for ULP distances)."""
    if a.dtype == np.float32:
        i = a.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)
    i = a.view(np.int64)
    mag = i & 0x7FFFFFFFFFFFFFFF
    return np.where(i < 0, -mag, mag)


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """ULP distance per element; NaN vs NaN counts 0, NaN vs number counts huge."""
    a = np.asarray(a)
    b = np.asarray(b)
    na, nb = np.isnan(a), np.isnan(b)
    d = np.abs(ordered_bits(a) - ordered_bits(b))
    d = np.where(na & nb, 0, d)
    d = np.where(na ^ nb, np.iinfo(np.int64).max, d)
    return d


def assert_bit_exact(got: np.ndarray, want: np.ndarray, what: str = "") -> None:
    """Bit-identical, except that any NaN matches any NaN (payloads differ
    between x86 and CUDA for NaNs created by an operation)."""
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    if got.dtype.kind == "f":
        gn, wn = np.isnan(got), np.isnan(want)
        assert np.array_equal(gn, wn), f"{what}: NaN positions differ"
        ib = got.view(np.int32 if got.dtype == np.float32 else np.int64)
        wb = want.view(np.int32 if want.dtype == np.float32 else np.int64)
        bad = (ib != wb) & ~gn
        if bad.any():
            k = np.flatnonzero(bad.reshape(-1))[:5]
            raise AssertionError(f"{what}: {bad.sum()} elements differ in bits, e.g. at {k}: "
                                 f"got {got.reshape(-1)[k]} want {want.reshape(-1)[k]}")
    else:
        assert np.array_equal(got, want), f"{what}: values differ"


def max_ulp(got: np.ndarray, want: np.ndarray) -> int:
    d = ulp_diff(got, want)
    return int(d.max()) if d.size else 0
