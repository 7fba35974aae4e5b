"""K-RED parity: sum / mean / max / argmax along an axis, reduce_broadcast_grad
and the fused un-broadcast, on the GPU through the C ABI, against the oracle.

Tolerances: integer sums, max and argmax are bit-exact (NaN and tie rules
included).  f32/f64 sums accumulate in f64 on the GPU, so per output
|gpu - ref| <= 1e-5 * sum|x| against the reference's sequential f32 fold, and
|gpu - exact| <= 1 ulp(exact) + n * 2^-53 * sum|x| against the exact sum.
Means are the sum divided by n in the element type, with the same bound / n."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact

pytestmark = pytest.mark.gpu


def rand(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.standard_normal(size=shape).astype(dtype)
    return rng.integers(-1000, 1000, size=shape).astype(dtype)


def check_sum(got, ref, x_abs_sum, exact):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape
    assert np.all(np.abs(got - ref) <= 1e-5 * x_abs_sum + 1e-30), float(np.max(np.abs(got - ref) - 1e-5 * x_abs_sum))
    tol = np.abs(exact) * 2.0**-23 + 2.0**-40 * x_abs_sum + 1e-300
    assert np.all(np.abs(got - exact) <= tol)


def axis_sums_f64(x: np.ndarray, axis, keepdim):
    xd = x.astype(np.float64)
    return xd.sum(axis=axis, keepdims=keepdim), np.abs(xd).sum(axis=axis, keepdims=keepdim)


SHAPES_AXES = [([1024, 1024], 0), ([1024, 1024], 1), ([7, 13, 5], 0), ([7, 13, 5], 1), ([7, 13, 5], 2),
               ([3, 300, 50], 1), ([64, 8, 3136], 2), ([4096, 65], 0), ([65, 4096], 1), ([1, 1], 0),
               ([20000], 0), ([2, 3, 4, 5, 6], 3), ([300000, 3], 0), ([3, 300000], 1)]


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,axis", SHAPES_AXES, ids=lambda v: str(v))
@pytest.mark.parametrize("keepdim", [False, True])
def test_sum_axis(shape, axis, keepdim, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, sum(shape) + axis)
    dx = contiguous(x)
    oshape = list(shape)
    if keepdim:
        oshape[axis] = 1
    else:
        oshape.pop(axis)
    got = to_host(device.sum_axis(dx.view, axis, keepdim, empty(oshape, dtype)))
    ref = oracle.sum_axis(dx.host_view(), axis, keepdim)
    if np.dtype(dtype).kind == "i":
        assert_bit_exact(got, ref)
    else:
        exact, sabs = axis_sums_f64(x, axis, keepdim)
        check_sum(got, ref, sabs, exact)


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,axis", [([1024, 1024], 1), ([33, 77], 0), ([8, 16384], 1), ([2048, 300], 0)])
def test_mean_axis(shape, axis, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, 3)
    dx = contiguous(x)
    oshape = list(shape)
    oshape[axis] = 1
    got = to_host(device.mean_axis(dx.view, axis, True, empty(oshape, dtype)))
    ref = oracle.mean_axis(dx.host_view(), axis, True)
    exact, sabs = axis_sums_f64(x, axis, True)
    n = shape[axis]
    check_sum(np.asarray(got, np.float64) * n, np.asarray(ref, np.float64) * n, sabs, exact)


def test_sum_axis_on_strided_views():
    import oracle
    from tensorrs_b200 import device
    st = rand([5000], np.float32, 4)
    for shape, strides, off, axis in [([40, 30], [1, 40], 0, 0), ([40, 30], [1, 40], 0, 1),
                                      ([20, 25], [-100, 3], 2000 + 99, 1), ([10, 10, 10], [7, 300, -1], 20, 2)]:
        dv = DevView(st, shape, strides, off)
        oshape = [s for i, s in enumerate(shape) if i != axis]
        got = to_host(device.sum_axis(dv.view, axis, False, empty(oshape, np.float32)))
        ref = oracle.sum_axis(dv.host_view(), axis, False)
        packed = oracle.unary("none", dv.host_view())
        exact, sabs = axis_sums_f64(packed, axis, False)
        check_sum(got, ref, sabs, exact)


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,axis", [([1024, 1024], 0), ([1024, 1024], 1), ([7, 13, 5], 1), ([8, 16384], 1),
                                        ([16384, 8], 0), ([3, 5, 300, 2], 2), ([1, 9], 1), ([300000], 0)])
def test_max_and_argmax_bit_exact(shape, axis, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, 9)
    if np.dtype(dtype).kind == "i":
        x = x % 50  # many ties
    else:
        x = np.round(x * 4) / 4  # many ties
    dx = contiguous(x)
    oshape = [s for i, s in enumerate(shape) if i != axis]
    vals = to_host(device.max_axis(dx.view, axis, empty(oshape, dtype)))
    idx = to_host(device.argmax_axis(dx.view, axis, empty(oshape, np.int64)))
    rv, ri = oracle.max_argmax_axis(dx.host_view(), axis)
    assert_bit_exact(vals, rv, "max")
    assert_bit_exact(idx, ri, "argmax")


def test_max_argmax_nan_and_signed_zero_rules():
    """strict `>` from the first element (base.rs:1404-1411, 1467-1478)."""
    import oracle
    from tensorrs_b200 import device
    nan, inf = np.nan, np.inf
    rows = [
        [nan, 1.0, 2.0, 3.0],     # NaN at index 0 sticks
        [1.0, nan, 2.0, nan],     # later NaNs never win
        [-0.0, 0.0, -0.0, 0.0],   # -0 == +0: the first one stays
        [0.0, -0.0, 0.0, 0.0],
        [nan, nan, nan, nan],
        [-inf, -inf, -inf, -inf],
        [-inf, nan, -inf, 5.0],
        [2.0, 2.0, 2.0, 1.0],
    ]
    x = np.array(rows, np.float32)
    # long rows too, so the parallel kernels combine partials
    big = np.tile(np.array(rows, np.float32), (1, 4096))
    for arr in (x, big, np.ascontiguousarray(big.T)):
        for axis in (0, 1):
            dx = contiguous(arr)
            oshape = [s for i, s in enumerate(arr.shape) if i != axis]
            vals = to_host(device.max_axis(dx.view, axis, empty(oshape, np.float32)))
            idx = to_host(device.argmax_axis(dx.view, axis, empty(oshape, np.int64)))
            rv, ri = oracle.max_argmax_axis(dx.host_view(), axis)
            assert_bit_exact(vals, rv)
            assert np.array_equal(np.signbit(vals), np.signbit(rv))
            assert_bit_exact(idx, ri)


def test_axis_errors_match_reference_panics():
    from tensorrs_b200 import abi, device
    dx = contiguous(np.zeros([3, 0], np.float32))
    with pytest.raises(abi.TrsError) as e:
        device.max_axis(dx.view, 1, empty([3], np.float32))
    assert "!!!Cannot reduce an empty axis!!!" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.sum_axis(dx.view, 2, False, empty([3], np.float32))
    assert "!!!Axis index out of range!!!" in e.value.message
    # an empty axis sums to zeros (sum_axis has no emptiness check)
    got = to_host(device.sum_axis(dx.view, 1, False, empty([3], np.float32)))
    assert np.array_equal(got, np.zeros(3, np.float32))


RBG_CASES = [
    ([2, 3], [3]), ([2, 3], [1, 3]), ([2, 3], [2, 1]), ([2, 3], [1, 1]), ([2, 2, 2], [2, 2]),
    ([2, 3], [2, 2]), ([2, 3], [2, 3]), ([1], [4, 5]), ([3], [2, 3]), ([64, 32, 14, 14], [1, 32, 1, 1]),
    ([128, 1000], [1000]), ([5, 6, 7], [6, 1]), ([8, 1, 9], [1, 1, 9]), ([4, 5], []),
]


@pytest.mark.parametrize("dtype", [np.float32, np.int32], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,target", RBG_CASES, ids=lambda v: str(v))
def test_reduce_broadcast_grad(shape, target, dtype):
    import oracle
    from tensorrs_b200 import abi, device
    g = rand(shape, dtype, 17)
    dg = contiguous(g)
    ref = oracle.reduce_broadcast_grad(dg.host_view(), target)
    out = empty(target if target else [1], dtype) if target else empty([], dtype)
    st = device.reduce_broadcast_grad(dg.view, target, out)
    if ref is None:
        assert st == abi.NONE
        return
    assert st == abi.OK
    got = to_host(out).reshape(ref.shape)
    if np.dtype(dtype).kind == "i":
        assert_bit_exact(got, ref)
    else:
        gd = g.astype(np.float64).reshape(shape)
        # exact sums over the broadcast axes
        exact = oracle.reduce_broadcast_grad(oracle.contiguous(gd), target)
        sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(gd)), target)
        check_sum(got, ref, sabs, exact)


def test_sum_to_shape_fused_equals_the_mul_backward_chain():
    """Mul backward (autodiff/core.rs:206-227): reduce_to_shape(g & mask & x)."""
    import oracle
    from tensorrs_b200 import device
    shape, target = [16, 32, 9, 11], [1, 32, 1, 1]
    g = rand(shape, np.float32, 21)
    pre = rand(shape, np.float32, 22)
    x = rand(shape, np.float32, 23)
    dg, dp, dx = contiguous(g), contiguous(pre), contiguous(x)
    mask = (pre > 0).astype(np.float32)
    gm = oracle.binary("mul", dg.host_view(), oracle.contiguous(mask))
    prod = oracle.binary("mul", oracle.contiguous(gm), dx.host_view())
    ref = oracle.reduce_broadcast_grad(oracle.contiguous(prod), target)
    out = empty(target, np.float32)
    device.sum_to_shape_fused(dg.view, dp.view, dx.view, target, out)
    got = to_host(out)
    exact = oracle.reduce_broadcast_grad(oracle.contiguous(prod.astype(np.float64)), target)
    sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(prod.astype(np.float64))), target)
    check_sum(got, ref, sabs, exact)
    # without gate and multiplicand it is reduce_broadcast_grad itself
    out2 = empty([32, 1, 1], np.float32)
    device.sum_to_shape_fused(dg.view, None, None, [32, 1, 1], out2)
    ref2 = oracle.reduce_broadcast_grad(dg.host_view(), [32, 1, 1])
    ex2 = oracle.reduce_broadcast_grad(oracle.contiguous(g.astype(np.float64)), [32, 1, 1])
    sa2 = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(g.astype(np.float64))), [32, 1, 1])
    check_sum(to_host(out2), ref2, sa2, ex2)


@pytest.mark.parametrize("shape", [[4, 16, 7, 9], [64, 256, 14, 14], [2, 8, 1, 1]])
def test_affine_relu_backward_equals_the_reference_chain(shape):
    """ReLU(x & s + b) backward: bias grad = reduce(g & m), scale grad = reduce((g & m) & x)."""
    import oracle
    from tensorrs_b200 import device
    c = shape[1]
    g = rand(shape, np.float32, 31)
    x = rand(shape, np.float32, 32)
    s = oracle.fill_uniform(np.float32, c, 3, 0.5, 1.5).reshape(1, c, 1, 1)
    b = oracle.fill_uniform(np.float32, c, 4, -0.1, 0.1).reshape(1, c, 1, 1)
    dg, dx, ds, db = contiguous(g), contiguous(x), contiguous(s), contiguous(b)
    z = oracle.program(3, "mul", "add", "none", [dx.host_view(), ds.host_view(), db.host_view()])
    mask = (z > 0).astype(np.float32)
    gm = oracle.binary("mul", dg.host_view(), oracle.contiguous(mask))
    gmx = oracle.binary("mul", oracle.contiguous(gm), dx.host_view())
    t = [1, c, 1, 1]
    ref_b = oracle.reduce_broadcast_grad(oracle.contiguous(gm), t)
    ref_s = oracle.reduce_broadcast_grad(oracle.contiguous(gmx), t)
    gs, gb = empty(t, np.float32), empty(t, np.float32)
    device.affine_relu_backward(dg.view, dx.view, ds.view, db.view, gs, gb)
    for got, ref, prod in [(to_host(gs), ref_s, gmx), (to_host(gb), ref_b, gm)]:
        pd = prod.astype(np.float64)
        exact = oracle.reduce_broadcast_grad(oracle.contiguous(pd), t)
        sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(pd)), t)
        check_sum(got, ref, sabs, exact)


@pytest.mark.parametrize("dtype", [np.float32, np.int64], ids=lambda d: np.dtype(d).name)
def test_full_sum(dtype):
    import oracle
    from tensorrs_b200 import device
    for shape in [[1024, 1024], [3, 7, 11], [1], [1 << 22]]:
        x = rand(shape, dtype, 41)
        dx = contiguous(x)
        got = to_host(device.sum_all(dx.view, empty([1], dtype)))[0]
        ref = oracle.sum_all(dx.host_view())
        if np.dtype(dtype).kind == "i":
            assert got == ref
        else:
            exact, sabs = oracle.sum_f64(dx.host_view())
            check_sum(np.array([got]), np.array([ref]), sabs, np.array([exact]))
