"""Host check of the f32 exponential the kernels use for sigmoid, ELU, SELU
and SoftMax (tensorrs_b200/csrc/exp_f32.h).

The header compiles unchanged for the host; tests/cpp/exp_check.cpp evaluates
its f32 operations with g++ under strict IEEE arithmetic (every step an
explicitly rounded add, multiply or fused multiply-add, as on the GPU) and
compares with glibc's expf(y) and powf(2.7182817f, y), the functions the
reference's Float::exp and powf call (src/lib.rs:148-160, via
activation/elu.rs:59-60 and activation/softmax.rs:59-61 for powf(E, .)).

Bounds (the transcendental tolerance is two ulp): at most one ulp from glibc
everywhere in the fast range [-86, 87] and bit-identical for at least 99 % of
the inputs of each range.  The branch-free form for y <= 0 (sigmoid, softmax)
covers every y from -0 to -inf and NaN: at most one ulp from glibc, NaN
exactly where glibc gives NaN, and equal to the fast path inside its range.
"""
from __future__ import annotations

import functools
import subprocess
from pathlib import Path

from conftest import ROOT

SRC = ROOT / "tests" / "cpp" / "exp_check.cpp"
BIN = ROOT / "tests" / "cpp" / "_build" / "exp_check"


def _build() -> Path:
    BIN.parent.mkdir(exist_ok=True)
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    cmd = [cxx, "-std=c++17", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wextra",
           "-I", str(ROOT / "tensorrs_b200" / "csrc"), str(SRC), "-o", str(BIN), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return BIN


@functools.lru_cache(maxsize=1)
def _rows() -> tuple[tuple[str, ...], ...]:
    out = subprocess.run([str(_build()), "13"], check=True, capture_output=True, text=True, timeout=600).stdout
    rows = tuple(tuple(line.split()) for line in out.strip().splitlines())
    assert len(rows) == 14
    return rows


def test_sigmoid_division_is_the_ieee_quotient():
    """sigmoid_div (Markstein's division with a one-ulp reciprocal seed and a
    floor on the refined reciprocal) equals num / (1 + e) rounded once, for
    every f32 e in [0, 1], both numerators and every seed within one ulp."""
    (row,) = [r for r in _rows() if r[0] == "sigmoid_div"]
    count, bad = int(row[3]), int(row[6])
    assert count == 6 * (0x3F800000 + 1)
    assert bad == 0


def test_sigmoid_within_two_ulp_of_the_reference_formula():
    """The whole f32 sigmoid (autodiff/ops.rs:586-593 on glibc's expf) over
    a strided sweep of every f32: NaN exactly where the reference gives NaN,
    at most two ulp apart, and bit-identical for at least 99.9 %."""
    (row,) = [r for r in _rows() if r[0] == "sigmoid"]
    count, same, worst, bad = int(row[3]), int(row[4]), int(row[5]), int(row[6])
    assert count > 100_000_000
    assert bad == 0
    assert worst <= 2
    assert same / count >= 0.999


def test_table_exponential_within_one_ulp_of_glibc():
    for name, lo, hi, count, same, worst, bad in _rows():
        if name.startswith("sigmoid"):
            continue
        count, same, worst, bad = int(count), int(same), int(worst), int(bad)
        assert count > 100_000, (name, lo, hi)
        assert bad == 0, (name, lo, hi, "outside the fast path, or unlike it")
        assert worst <= 1, (name, lo, hi, worst)
        assert same / count >= 0.99, (name, lo, hi, same / count)
