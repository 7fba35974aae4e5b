"""The element-wise bulk-copy pipeline (ew_stream_kernel), which takes
element-wise calls of at least 16 MiB with rows of at least 4 KiB: every
compiled program it carries (A & B + c, ReLU(X & s + b), a op b, x, the
runtime-op fallbacks), inputs staged by bulk copies and inputs constant along
a row (per-row scalars), rows cut into several tiles with a short last one,
all dtypes, the sum epilogue with and without the written output.  Bit-exact
against the oracle; sums within the bounds of test_reduce_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import contiguous, empty, to_host
from _util import assert_bit_exact

pytestmark = pytest.mark.gpu


def rand(shape, dtype, seed, lo=-2.0, hi=2.0):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.uniform(lo, hi, size=shape).astype(dtype)
    return rng.integers(-1000, 1000, size=shape).astype(dtype)


def _check_sum(got, want_arr):
    """Against the exact sum: 1 ulp + n * 2^-40 * sum|x|.  Against the
    reference's sequential f32 fold: 1e-5 * sum|x|, or the fold's own error
    bound (n - 1) * 2^-24 * sum|x| where that is larger (a long sum of
    non-negative terms, such as ReLU outputs, drifts far beyond 1e-5)."""
    import oracle
    ref = oracle.sum_all(oracle.contiguous(want_arr))
    exact, sabs = oracle.sum_f64(oracle.contiguous(want_arr))
    n = want_arr.size
    assert abs(float(got) - exact) <= abs(exact) * 2.0**-23 + 2.0**-40 * sabs
    assert abs(float(got) - float(ref)) <= max(1e-5, (n - 1) * 2.0**-24) * sabs


CASES = [
    # (name, n_in, op1, op2, epilogue, shapes)
    ("fma_sum config-5 layout", 3, "mul", "add", "none", [[2048, 8192], [2048, 8192], [8192]]),
    ("relu affine config-4 layout", 3, "mul", "add", "relu", [[16, 256, 56, 56], [1, 256, 1, 1], [1, 256, 1, 1]]),
    ("add with row bias", 2, "add", "add", "none", [[2048, 4096], [4096]]),
    ("sub with per-row scalar", 2, "sub", "add", "none", [[2048, 4096], [2048, 1]]),
    ("mul", 2, "mul", "add", "none", [[2048, 4096], [2048, 4096]]),
    ("div", 2, "div", "add", "none", [[2048, 4096], [2048, 4096]]),
    ("split tiles (rows of 5000)", 2, "add", "add", "none", [[1024, 5000], [1024, 5000]]),
    ("runtime ops with a scalar epilogue", 3, "sub", "mul", "clamp", [[1024, 8192], [8192], [1024, 1]]),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0])
def test_stream_programs_bit_exact(case):
    import oracle
    from tensorrs_b200 import abi, device
    name, n_in, op1, op2, epi, shapes = case
    arrs = [rand(s, np.float32, 60 + i) for i, s in enumerate(shapes)]
    if op1 == "div":
        arrs[1][np.abs(arrs[1]) < 0.1] = 0.5
    dvs = [contiguous(a) for a in arrs]
    p0, p1 = (-1.0, 1.5) if epi == "clamp" else (0.0, 0.0)
    want = oracle.program(n_in, op1, op2, epi, [d.host_view() for d in dvs], p0, p1)
    out = empty(want.shape, np.float32)
    s = empty([1], np.float32)
    prog = abi.program(n_in, abi.BINOPS[op1], abi.BINOPS[op2], epi, p0, p1)
    device.elementwise(prog, [d.view for d in dvs], out, s)
    assert_bit_exact(to_host(out), want, name)
    _check_sum(to_host(s)[0], want)


@pytest.mark.parametrize("dtype", [np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
def test_stream_other_dtypes(dtype):
    import oracle
    from tensorrs_b200 import device
    a = rand([2048, 2048], dtype, 70)
    b = rand([2048], dtype, 71)
    da, db = contiguous(a), contiguous(b)
    want = oracle.binary("add", da.host_view(), db.host_view())
    assert_bit_exact(to_host(device.binary("add", da.view, db.view, empty([2048, 2048], dtype))), want)


def test_stream_pack_and_sum_only():
    """x packed (kPack) and sum(x) with no written output (the sum epilogue
    alone), 64 MiB."""
    import oracle
    from tensorrs_b200 import device
    x = rand([4096, 4096], np.float32, 72)
    dx = contiguous(x)
    assert_bit_exact(to_host(device.pack(dx.view, empty([4096, 4096], np.float32))), x)
    got = to_host(device.sum_all(dx.view, empty([1], np.float32)))[0]
    _check_sum(got, x)


def test_no_stream_kernel_gave_up_waiting_on_its_copies():
    import ctypes

    from tensorrs_b200 import abi
    code = ctypes.c_int32(-1)
    abi.check(abi.load().trs_async_error(ctypes.byref(code)))
    assert code.value == 0
