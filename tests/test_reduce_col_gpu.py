"""Column reductions (the reduced rows run across the contiguous kept
dimension W: sum_axis(0) of a row-major matrix, the leading-axis un-broadcast
of reduce_broadcast_grad) on the bulk-copy column pipeline, against the
oracle.  Shapes cover: one and several column blocks (a block is 2 KiB of a
row), a narrower last block, W that is not a power of two, row counts that
are not a multiple of the rows staged per step, several outer kept indices,
several reduced dimensions, and outputs split into row parts.

Tolerances as in test_reduce_gpu.py: integer sums, max and argmax bit-exact;
float sums within 1e-5 * sum|x| of the reference's sequential fold and within
1 ulp + n * 2^-40 * sum|x| of the exact sum."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import contiguous, empty, to_host
from _util import assert_bit_exact
from test_reduce_gpu import axis_sums_f64, check_sum, rand

pytestmark = pytest.mark.gpu

COL_CASES = [([1024, 1024], 0), ([4096, 2048], 0), ([3000, 1000], 0), ([2048, 300], 0), ([513, 4096], 0),
             ([8192, 512], 0), ([64, 256, 1024], 1), ([256, 4, 1024], 0), ([700, 3, 640], 0)]


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,axis", COL_CASES, ids=lambda v: str(v))
def test_column_sum(shape, axis, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, sum(shape) + 5)
    dx = contiguous(x)
    oshape = [s for i, s in enumerate(shape) if i != axis]
    got = to_host(device.sum_axis(dx.view, axis, False, empty(oshape, dtype)))
    ref = oracle.sum_axis(dx.host_view(), axis, False)
    if np.dtype(dtype).kind == "i":
        assert_bit_exact(got, ref)
    else:
        exact, sabs = axis_sums_f64(x, axis, False)
        check_sum(got, ref, sabs, exact)


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape", [[4096, 2048], [1500, 700]], ids=str)
def test_column_mean(shape, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, 8)
    dx = contiguous(x)
    got = to_host(device.mean_axis(dx.view, 0, True, empty([1, shape[1]], dtype)))
    ref = oracle.mean_axis(dx.host_view(), 0, True)
    exact, sabs = axis_sums_f64(x, 0, True)
    n = shape[0]
    check_sum(np.asarray(got, np.float64) * n, np.asarray(ref, np.float64) * n, sabs, exact)


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,axis", [([4096, 2048], 0), ([3000, 1000], 0), ([513, 4096], 0),
                                        ([64, 256, 1024], 1)], ids=lambda v: str(v))
def test_column_max_argmax(shape, axis, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, 13)
    x = (x % 40) if np.dtype(dtype).kind == "i" else np.round(x * 3) / 3  # many ties
    if np.dtype(dtype).kind == "f" and axis == 0:
        x[0, 3] = np.nan            # NaN at index 0 sticks
        x[7, 4] = np.nan            # later NaN never wins
        x[:, 5] = -np.inf           # all -inf: index 0
        x[:, 6] = np.nan            # all NaN
        x[-1, 6] = 1.0
        x[:, 7] = 0.0
        x[3, 7] = -0.0
        x[0, 7] = -0.0              # -0 first: stays
        x[:, 8] = 2.0               # one value everywhere: index 0
        x[shape[0] - 1, 9] = 100.0  # the maximum in the last row of the last part
        x[shape[0] // 2, 10] = 100.0
        x[shape[0] // 2 + 1, 10] = 100.0
    dx = contiguous(x)
    oshape = [s for i, s in enumerate(shape) if i != axis]
    vals = to_host(device.max_axis(dx.view, axis, empty(oshape, dtype)))
    idx = to_host(device.argmax_axis(dx.view, axis, empty(oshape, np.int64)))
    rv, ri = oracle.max_argmax_axis(dx.host_view(), axis)
    assert_bit_exact(vals, rv, "max")
    if np.dtype(dtype).kind == "f":
        assert np.array_equal(np.signbit(vals), np.signbit(rv))
    assert_bit_exact(idx, ri, "argmax")


@pytest.mark.parametrize("dtype", [np.float32, np.int32], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,target", [([64, 32, 2048], [2048]), ([8, 64, 1000], [1, 1, 1000]),
                                          ([16, 300, 512], [1, 512]), ([4096, 1024], [1, 1024])],
                         ids=lambda v: str(v))
def test_column_reduce_broadcast_grad(shape, target, dtype):
    import oracle
    from tensorrs_b200 import abi, device
    g = rand(shape, dtype, 19)
    dg = contiguous(g)
    ref = oracle.reduce_broadcast_grad(dg.host_view(), target)
    out = empty(target, dtype)
    assert device.reduce_broadcast_grad(dg.view, target, out) == abi.OK
    got = to_host(out).reshape(ref.shape)
    if np.dtype(dtype).kind == "i":
        assert_bit_exact(got, ref)
    else:
        gd = g.astype(np.float64)
        exact = oracle.reduce_broadcast_grad(oracle.contiguous(gd), target)
        sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(gd)), target)
        check_sum(got, ref, sabs, exact)


@pytest.mark.parametrize("mul_shape", [[4096, 1024], [1, 1024], [4096, 1]], ids=str)
def test_column_sum_to_shape_fused(mul_shape):
    """Mul backward un-broadcast (autodiff/core.rs:206-227) of a [rows, W]
    gradient to [1, W], with the multiplicand full, broadcast along rows, or
    constant along W."""
    import oracle
    from tensorrs_b200 import device
    shape, target = [4096, 1024], [1, 1024]
    g = rand(shape, np.float32, 51)
    pre = rand(shape, np.float32, 52)
    m = rand(mul_shape, np.float32, 53)
    dg, dp, dm = contiguous(g), contiguous(pre), contiguous(m)
    mask = (pre > 0).astype(np.float32)
    gm = oracle.binary("mul", dg.host_view(), oracle.contiguous(mask))
    prod = oracle.binary("mul", oracle.contiguous(gm), dm.host_view())
    ref = oracle.reduce_broadcast_grad(oracle.contiguous(prod), target)
    out = empty(target, np.float32)
    device.sum_to_shape_fused(dg.view, dp.view, dm.view, target, out)
    pd = prod.astype(np.float64)
    exact = oracle.reduce_broadcast_grad(oracle.contiguous(pd), target)
    sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(pd)), target)
    check_sum(to_host(out), ref, sabs, exact)


def test_column_reductions_config3_full_size():
    """sum_axis(0), max_axis(0) and argmax_axis(0) of X f32 [8192, 16384] ~N(0,1)."""
    import oracle
    from tensorrs_b200 import device
    x = oracle.fill_normal(np.float32, 8192 * 16384, 2).reshape(8192, 16384)
    dx = contiguous(x)
    got = to_host(device.sum_axis(dx.view, 0, False, empty([16384], np.float32)))
    ref = oracle.sum_axis(dx.host_view(), 0, False)
    exact, sabs = axis_sums_f64(x, 0, False)
    check_sum(got, ref, sabs, exact)
    vals = to_host(device.max_axis(dx.view, 0, empty([16384], np.float32)))
    idx = to_host(device.argmax_axis(dx.view, 0, empty([16384], np.int64)))
    rv, ri = oracle.max_argmax_axis(dx.host_view(), 0)
    assert_bit_exact(vals, rv, "max")
    assert_bit_exact(idx, ri, "argmax")


def test_no_column_kernel_gave_up_waiting_on_its_copies():
    """Every bulk-copy wait of the runs above completed (none hit its bound)."""
    import ctypes

    from tensorrs_b200 import abi
    code = ctypes.c_int32(-1)
    abi.check(abi.load().trs_async_error(ctypes.byref(code)))
    assert code.value == 0
