"""Gradient accumulation and zero_grad on the device, as AutoGrad::backward and
AutoGrad::zero_grad do them (autodiff/traits.rs:55-71, 122-152), through the
C ABI against the oracle's chain.

  * accumulation: `current + grad_to_add` (traits.rs:148) written back over the
    current gradient -- trs_binary(ADD, cur, grad, out = cur), the output
    aliasing its first input through the identical layout;
  * the fallback when a parent's gradient has a broadcast shape: reduce it to
    the expected shape first (traits.rs:124-139, reduce_to_shape ->
    reduce_broadcast_grad), then add; a shape that is not a broadcast of the
    expected one is the reference's None, after which the caller tries the
    parent's value shape;
  * zero_grad: `full_(T::default())` -- trs_pack from a zero-stride view of a
    single +0 (every element +0, whatever it held, -0 and NaN included).

Element-wise results are bit-exact; the reduction in the fallback is a sum
(f64 accumulation, rounded once) and is held to the sum tolerance of
test_reduce_gpu.py, after which the addition is bit-exact again."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact

pytestmark = pytest.mark.gpu

DTYPES = [np.float32, np.float64, np.int32, np.int64]


def rand(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.standard_normal(size=shape).astype(dtype)
    return rng.integers(-1000, 1000, size=shape).astype(dtype)


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape", [[1], [7, 13], [256, 1024], [3, 5, 7, 11], [1 << 22]])
def test_in_place_accumulation_of_several_gradients(shape, dtype):
    """Three backward contributions added one after another into the same
    gradient buffer, as a node with three consumers receives them."""
    import oracle
    from tensorrs_b200 import abi
    lib = abi.load()
    cur = rand(shape, dtype, 1)
    dc = contiguous(cur)
    want = cur.copy()
    for k in range(3):
        g = rand(shape, dtype, 10 + k)
        dg = contiguous(g)
        v = dc.view
        abi.check(lib.trs_binary(abi.ADD, ctypes.byref(v), ctypes.byref(dg.view), ctypes.byref(v),
                                 _stream()))
        want = oracle.binary("add", oracle.contiguous(want), dg.host_view())
    assert_bit_exact(to_host(dc.t).reshape(shape), want, "accumulated gradient")


def _stream():
    from tensorrs_b200 import device
    return device.stream_handle()


@pytest.mark.parametrize("dtype", [np.float32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("grad_shape,expected", [([64, 256], [256]), ([64, 256], [1, 256]),
                                                 ([8, 32, 14, 14], [1, 32, 1, 1]), ([5, 6, 7], [6, 1])])
def test_broadcast_gradient_reduced_then_accumulated(grad_shape, expected, dtype):
    import oracle
    from tensorrs_b200 import abi, device
    lib = abi.load()
    g = rand(grad_shape, dtype, 3)
    cur = rand(expected, dtype, 4)
    dg, dc = contiguous(g), contiguous(cur)
    red = empty(expected, dtype)
    assert device.reduce_broadcast_grad(dg.view, expected, red) == abi.OK
    got_red = to_host(red)
    ref_red = oracle.reduce_broadcast_grad(dg.host_view(), expected)
    if np.dtype(dtype).kind == "i":
        assert_bit_exact(got_red, ref_red, "reduced gradient")
    else:
        gd = g.astype(np.float64)
        exact = oracle.reduce_broadcast_grad(oracle.contiguous(gd), expected)
        sabs = oracle.reduce_broadcast_grad(oracle.contiguous(np.abs(gd)), expected)
        assert np.all(np.abs(got_red.astype(np.float64) - ref_red) <= 1e-5 * sabs + 1e-30)
        assert np.all(np.abs(got_red.astype(np.float64) - exact) <= np.abs(exact) * 2.0**-23 + 2.0**-40 * sabs)
    v = dc.view
    abi.check(lib.trs_binary(abi.ADD, ctypes.byref(v), ctypes.byref(device.view_of(red)),
                             ctypes.byref(v), _stream()))
    want = oracle.binary("add", dc.host_view(), oracle.contiguous(got_red))
    assert_bit_exact(to_host(dc.t).reshape(expected), want, "accumulated reduced gradient")


def test_fallback_order_when_the_expected_shape_is_not_a_broadcast_target():
    """[2, 3] cannot be reduced to [2, 2] (None, traits.rs:129); the caller then
    reduces to the parent's value shape, here [3]."""
    import oracle
    from tensorrs_b200 import abi, device
    g = rand([2, 3], np.float32, 5)
    dg = contiguous(g)
    assert device.reduce_broadcast_grad(dg.view, [2, 2], empty([2, 2], np.float32)) == abi.NONE
    assert oracle.reduce_broadcast_grad(dg.host_view(), [2, 2]) is None
    out = empty([3], np.float32)
    assert device.reduce_broadcast_grad(dg.view, [3], out) == abi.OK
    ref = oracle.reduce_broadcast_grad(dg.host_view(), [3])
    gd = g.astype(np.float64)
    got = to_host(out).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * np.abs(gd).sum(axis=0) + 1e-30)
    assert np.all(np.abs(got - gd.sum(axis=0)) <= np.abs(gd.sum(axis=0)) * 2.0**-23 + 2.0**-40 * np.abs(gd).sum(axis=0))


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape", [[1], [33, 65], [4, 256, 56, 56]])
def test_zero_grad_fills_positive_zero(shape, dtype):
    from tensorrs_b200 import device
    n = int(np.prod(shape))
    junk = rand(shape, dtype, 6)
    if np.dtype(dtype).kind == "f":
        flat = junk.reshape(-1)
        flat[: min(n, 4)] = np.array([-0.0, np.nan, -np.inf, 1.0], dtype)[: min(n, 4)]
    grad = contiguous(junk)
    zero = DevView(np.zeros(1, dtype), shape, [0] * len(shape), 0)
    device.pack(zero.view, grad.t.view(shape))
    got = to_host(grad.t)
    assert_bit_exact(got, np.zeros(n, dtype), "zero_grad")
    if np.dtype(dtype).kind == "f":
        assert not np.signbit(got).any()
