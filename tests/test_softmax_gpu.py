"""K-SOFTMAX parity against SoftMax::forward (activation/softmax.rs:42-68).

Each output is e / s with e = powf(E, x - max) and s the row sum.  The GPU's
e is within k_e ulp of the oracle's e_ref (1 ulp for f32, measured by the
dense sweep in test_ew_gpu.py; 4 for f64, CUDA's pow against glibc's), its
sum is accumulated in f64 and rounded once, and the quotient is rounded once.
So against ideal = e_ref / s_exact (the oracle's e, exactly summed):
  |got - ideal| <= ulp(ideal) + k_e * ulp(e_ref) / s_exact
                   + ideal * (2^-p + (n - 1) * 2^-53)
(p = 24 or 53: the rounding of the sum).  Against the reference itself the
reference's own sequential-sum error comes on top."""
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
    k_e = 1 if dt == np.float32 else 4
    p_rel = 2.0**-24 if dt == np.float32 else 2.0**-53
    with np.errstate(invalid="ignore"):
        tol_ideal = (np.spacing(np.abs(ideal).astype(dt)).astype(np.float64)
                     + k_e * np.spacing(np.abs(e)).astype(np.float64) / s_exact
                     + np.abs(ideal) * (p_rel + sum_rel))
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


@pytest.mark.parametrize("cols", [1024, 4096, 16384, 20000])
def test_softmax_special_rows_on_the_staged_path(cols):
    """Rows staged through shared memory: NaN at index 0 (the row is NaN), a
    later NaN (the sum is NaN), -inf rows (x - max is NaN), +inf, a -0/+0
    maximum, one dominant value, and ordinary rows around them."""
    import oracle
    from tensorrs_b200 import device
    rng = np.random.default_rng(cols)
    x = (rng.standard_normal((12, cols)) * 4).astype(np.float32)
    x[1, 0] = np.nan
    x[2, 7] = np.nan
    x[3, :] = -np.inf
    x[4, 5] = np.inf
    x[5, :] = -1.0
    x[5, 3] = -0.0
    x[5, 9] = 0.0
    x[6, :] = 0.0
    x[6, 0] = -0.0
    x[7, cols // 2] = 1000.0
    x[8, :] = np.nan
    x[9, :] = -100.0         # uniform row
    x[10, ::2] = -120.0      # exponents far below the f32 range: e = 0
    dx = contiguous(x)
    got = to_host(device.softmax_lastdim(dx.view, empty(x.shape, np.float32)))
    ref = oracle.softmax_lastdim(dx.host_view())
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    ok_rows = [i for i in range(x.shape[0]) if not np.isnan(ref[i]).any()]
    check_softmax(contiguous(np.ascontiguousarray(x[ok_rows])).host_view(), got[ok_rows])


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_softmax_config3_full_size(dtype):
    """X [8192, 16384] ~N(0,1) (the softmax workload; 2048 rows for f64)."""
    import oracle
    from tensorrs_b200 import device
    x = oracle.fill_normal(np.float32, 8192 * 16384, 2).reshape(8192, 16384).astype(dtype)
    if dtype == np.float64:
        x = np.ascontiguousarray(x[:2048])
    dx = contiguous(x)
    got = to_host(device.softmax_lastdim(dx.view, empty(x.shape, dtype)))
    check_softmax(dx.host_view(), got)


def test_no_kernel_gave_up_waiting_on_its_copies():
    """Every bulk-copy wait of the runs above completed (none hit its bound)."""
    import ctypes

    from tensorrs_b200 import abi
    code = ctypes.c_int32(-1)
    abi.check(abi.load().trs_async_error(ctypes.byref(code)))
    assert code.value == 0
