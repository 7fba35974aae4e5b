"""K-SOFTMAX parity against SoftMax::forward (activation/softmax.rs:42-68).

Each output is e / s with e = powf(E, x - max) and s the row sum.  The e
values agree with the oracle's to 2 ulp; the GPU sums in f64 while the
reference folds in f32, so against the reference each output may also differ
by the reference's own relative summation error.  Against e_ref / s_exact
(the same e, exactly summed) the GPU is within 3 ulp."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host

pytestmark = pytest.mark.gpu


def check_softmax(x_host_view, got):
    import math

    import oracle
    ref = oracle.softmax_lastdim(x_host_view)
    packed = oracle.unary("none", x_host_view)
    dt = packed.dtype
    axis = packed.ndim - 1
    mx, _ = oracle.max_argmax_axis(oracle.contiguous(packed), axis)
    shifted = oracle.binary("sub", oracle.contiguous(packed), oracle.contiguous(np.expand_dims(mx, -1)))
    e = oracle.unary("exp", oracle.contiguous(shifted))
    s_seq = oracle.sum_axis(oracle.contiguous(e), axis, True).astype(np.float64)
    rows = e.reshape(-1, e.shape[-1]).astype(np.float64)
    s_exact = np.array([math.fsum(r) for r in rows]).reshape(s_seq.shape)
    n = e.shape[-1]
    ideal = e.astype(np.float64) / s_exact
    # the GPU sums in f64: relative error <= (n-1) * 2^-53 (recursive summation)
    sum_rel = (n - 1) * 2.0**-53
    tol_ideal = 3 * np.spacing(np.abs(ideal).astype(dt)).astype(np.float64) + np.abs(ideal) * sum_rel
    finite = np.isfinite(ref)
    assert np.all(np.abs(got.astype(np.float64) - ideal)[finite] <= tol_ideal[finite])
    # against the reference: its own f32/f64 sequential-sum error on top
    rel = np.abs(s_seq - s_exact) / s_exact
    tol = np.abs(ref.astype(np.float64)) * (rel + sum_rel + 4 * np.finfo(dt).eps)
    assert np.all(np.abs(got.astype(np.float64) - ref.astype(np.float64))[finite] <= tol[finite] + 1e-300)
    assert np.array_equal(np.isnan(got), np.isnan(ref))


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 3), (100, 31), (64, 128), (33, 129), (17, 1000), (8, 1024),
                                       (4, 1025), (16, 4096), (8, 16384), (3, 20000), (2, 70001)])
def test_softmax_rows(rows, cols, dtype):
    from tensorrs_b200 import device
    rng = np.random.default_rng(rows * 7 + cols)
    x = (rng.standard_normal((rows, cols)) * 3).astype(dtype)
    dx = contiguous(x)
    got = to_host(device.softmax_lastdim(dx.view, empty(x.shape, dtype)))
    check_softmax(dx.host_view(), got)


def test_softmax_strided_and_special_rows():
    from tensorrs_b200 import device
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, 300)) * 5).astype(np.float32)
    x[1, 0] = np.nan          # NaN at index 0: the max is NaN, the row is NaN
    x[2, 7] = np.nan          # NaN later: the sum is NaN, the row is NaN
    x[3, :] = 0.0             # uniform row
    x[4, 5] = 1000.0          # one dominant value
    x[5, :] = -np.inf         # exponent of -inf - -inf is NaN
    dx = contiguous(x)
    got = to_host(device.softmax_lastdim(dx.view, empty(x.shape, np.float32)))
    import oracle
    ref = oracle.softmax_lastdim(dx.host_view())
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    finite_rows = [i for i in range(x.shape[0]) if not np.isnan(ref[i]).any()]
    check_softmax(contiguous(np.ascontiguousarray(x[finite_rows])).host_view(), got[finite_rows])
    # transposed view: rows are columns of the storage
    st = (rng.standard_normal(200 * 64)).astype(np.float32)
    dv = DevView(st, [64, 200], [1, 64], 0)
    got = to_host(device.softmax_lastdim(dv.view, empty([64, 200], np.float32)))
    check_softmax(dv.host_view(), got)


def test_softmax_rank3():
    from tensorrs_b200 import device
    rng = np.random.default_rng(4)
    x = rng.standard_normal((4, 6, 50)).astype(np.float32)
    dx = contiguous(x)
    got = to_host(device.softmax_lastdim(dx.view, empty(x.shape, np.float32)))
    check_softmax(dx.host_view(), got)


def test_no_kernel_gave_up_waiting_on_its_copies():
    """Every bulk-copy wait of the runs above completed (none hit its bound)."""
    import ctypes

    from tensorrs_b200 import abi
    code = ctypes.c_int32(-1)
    abi.check(abi.load().trs_async_error(ctypes.byref(code)))
    assert code.value == 0
