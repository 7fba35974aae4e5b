"""Tensor::matmul (linalg/tensor/base.rs:896-1013) and the im2col pair
unfold_2d / fold_2d (linalg/tensor/conv.rs:360-488) on the GPU through the C
ABI, against the oracle's restatements.

matmul keeps the reference's per-output chain acc = acc + a * b over k in
order from 0, each step rounded once in the element type, so every dtype is
compared bit for bit (integers wrap as in the reference's release build).
unfold is a gather and fold adds each pixel's windows in the reference's
order from +0: both bit-exact too."""
from __future__ import annotations

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
    # integers large enough that products and sums wrap in i32
    return rng.integers(-60000, 60000, size=shape).astype(dtype)


def gpu_matmul(da: DevView, db: DevView, dtype):
    from tensorrs_b200 import device
    out = empty(device.matmul_shape(da.view, db.view), dtype)
    return to_host(device.matmul(da.view, db.view, out))


MM_SHAPES = [
    ([1, 1], [1, 1]), ([3, 5], [5, 7]), ([17, 1], [1, 33]), ([129, 130], [130, 257]), ([64, 16], [16, 128]),
    ([256, 512], [512, 384]), ([1, 1000], [1000, 1]), ([5, 0], [0, 4]), ([0, 3], [3, 2]), ([2, 2, 2], [2, 2]),
    ([2, 1, 3, 20, 12], [4, 1, 12, 9]), ([7, 31, 40], [7, 40, 50]), ([3, 1, 8, 8], [1, 5, 8, 8]),
]


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("sa,sb", MM_SHAPES, ids=lambda v: str(v))
def test_matmul_bit_exact(sa, sb, dtype):
    import oracle
    a = rand(sa, dtype, sum(sa) + 1)
    b = rand(sb, dtype, sum(sb) + 2)
    da, db = contiguous(a), contiguous(b)
    want = oracle.matmul(da.host_view(), db.host_view())
    assert_bit_exact(gpu_matmul(da, db, dtype), want, f"matmul {sa} x {sb}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int64], ids=lambda d: np.dtype(d).name)
def test_matmul_through_views(dtype):
    """Transposed operands (A^T, B^T as strided views), an offset, a reversed
    (negative-stride) row order and a gapped row stride, each read through
    its strides as the reference reads them."""
    import oracle
    m, k, n = 70, 45, 90
    a_t = rand([k, m], dtype, 3)  # A = a_t^T
    b_t = rand([n, k], dtype, 4)  # B = b_t^T
    da = DevView(a_t, [m, k], [1, m], 0)
    db = DevView(b_t, [k, n], [1, k], 0)
    assert_bit_exact(gpu_matmul(da, db, dtype), oracle.matmul(da.host_view(), db.host_view()), "A^T x B^T")
    # A with an offset and a gapped row stride; B with its rows reversed
    store_a = rand([m * (k + 3) + 5], dtype, 5)
    da2 = DevView(store_a, [m, k], [k + 3, 1], 5)
    store_b = rand([k * n], dtype, 6)
    db2 = DevView(store_b, [k, n], [-n, 1], (k - 1) * n)
    assert_bit_exact(gpu_matmul(da2, db2, dtype), oracle.matmul(da2.host_view(), db2.host_view()), "strided")


def test_matmul_linear_layer_shape():
    """Linear::forward (nn/linear.rs:90-97): x [B, in] times W^T, W [out, in]
    read as a transposed view, at a size where the K chain is long."""
    import oracle
    x = rand([512, 1024], np.float32, 7)
    w = rand([768, 1024], np.float32, 8)
    dx = contiguous(x)
    dw = DevView(w, [1024, 768], [1, 1024], 0)
    assert_bit_exact(gpu_matmul(dx, dw, np.float32), oracle.matmul(dx.host_view(), dw.host_view()), "x W^T")


def test_matmul_special_values():
    """-0 products (acc starts at +0, so an all -0 chain gives +0 as in the
    reference), infinities and NaNs propagate through the same chain."""
    import oracle
    a = np.array([[-0.0, 1.0, np.inf], [2.0, np.nan, -1.0], [-0.0, -0.0, -0.0]], np.float32)
    b = np.array([[1.0, 0.0], [0.0, 2.0], [-0.0, 3.0]], np.float32)
    da, db = contiguous(a), contiguous(b)
    got = gpu_matmul(da, db, np.float32)
    want = oracle.matmul(da.host_view(), db.host_view())
    assert_bit_exact(got, want, "specials")
    assert not np.signbit(got[2, 0])


def test_matmul_errors_carry_the_reference_panic_text():
    from tensorrs_b200 import abi, device
    a = contiguous(np.ones([2, 3], np.float32))
    with pytest.raises(abi.TrsError) as e:
        device.matmul(contiguous(np.ones([3], np.float32)).view, a.view, empty([2, 3], np.float32))
    assert "matmul: both tensors must be at least 2D" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.matmul(a.view, a.view, empty([2, 3], np.float32))
    assert "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.matmul(contiguous(np.ones([2, 2, 3], np.float32)).view,
                      contiguous(np.ones([3, 3, 4], np.float32)).view, empty([3, 2, 4], np.float32))
    assert "matmul: batch shapes not broadcastable" in e.value.message
    with pytest.raises(abi.TrsError) as e:  # output of the wrong shape
        device.matmul(a.view, contiguous(np.ones([3, 4], np.float32)).view, empty([2, 5], np.float32))
    assert e.value.status == abi.ERR_SHAPE


def test_matmul_large_square():
    """[1024, 1024] x [1024, 1024] f32: every one of the 2^20 outputs is a
    1024-step chain, bit for bit."""
    import oracle
    a = rand([1024, 1024], np.float32, 9)
    b = rand([1024, 1024], np.float32, 10)
    da, db = contiguous(a), contiguous(b)
    assert_bit_exact(gpu_matmul(da, db, np.float32), oracle.matmul(da.host_view(), db.host_view()), "1024^3")


COL_CASES = [  # shape, kernel, stride, padding
    ([1, 1, 3, 3], (2, 2), (1, 1), (0, 0)), ([2, 3, 9, 11], (3, 3), (1, 1), (1, 1)),
    ([2, 3, 9, 11], (3, 2), (2, 3), (0, 1)), ([1, 4, 8, 8], (1, 1), (1, 1), (0, 0)),
    ([3, 2, 7, 5], (5, 5), (2, 2), (2, 2)), ([2, 16, 14, 14], (3, 3), (2, 2), (1, 1)),
    ([1, 1, 4, 4], (4, 4), (3, 3), (0, 0)), ([1, 2, 5, 6], (2, 3), (1, 1), (3, 2)),
    # more than 16 windows cover a pixel: fold adds them as it loads them
    ([1, 2, 9, 9], (5, 5), (1, 1), (2, 2)), ([2, 1, 12, 7], (7, 3), (1, 1), (3, 1)),
    # a row of exactly 2048 columns (the largest column table) and one of 2160 (past it)
    ([1, 128, 5, 6], (4, 4), (1, 1), (1, 1)), ([1, 240, 6, 7], (3, 3), (1, 1), (1, 1)),
    # fold windows too wide for a shared-memory tile: the per-pixel kernels
    ([1, 1, 6, 1200], (4, 4), (1, 1), (0, 0)), ([1, 1, 12, 20], (11, 11), (1, 1), (0, 0)),
    # unfold by output rows: a last channel block that is partial (70 = 24 + 24 + 22 channels) and
    # blocks rounded up to whole 16-byte stores (36 = 12 + 12 + 12)
    ([2, 70, 6, 40], (3, 3), (1, 1), (1, 1)), ([1, 36, 4, 100], (3, 3), (1, 1), (1, 1)),
    # stride-1 fold from TMA-staged window rows: strips of 64 columns, a partial channel block,
    # window rows above the image (no padding) that are zero-filled instead of copied
    ([1, 8, 5, 300], (3, 3), (1, 1), (1, 1)), ([2, 12, 9, 10], (3, 3), (1, 1), (1, 1)),
    ([2, 4, 8, 8], (3, 3), (1, 1), (0, 0)),
]


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape,kernel,stride,padding", COL_CASES, ids=lambda v: str(v))
def test_unfold_and_fold_bit_exact(shape, kernel, stride, padding, dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand(shape, dtype, sum(shape))
    dx = contiguous(x)
    want = oracle.unfold_2d(dx.host_view(), kernel, stride, padding)
    cols = device.unfold_2d(dx.view, kernel, stride, padding, empty(want.shape, dtype))
    assert_bit_exact(to_host(cols), want, "unfold_2d")
    # fold of independent values (each overlap sums distinct numbers)
    c = rand(want.shape, dtype, sum(shape) + 1)
    dc = contiguous(c)
    back = to_host(device.fold_2d(dc.view, kernel, stride, padding, empty(shape, dtype)))
    assert_bit_exact(back, oracle.fold_2d(dc.host_view(), shape, kernel, stride, padding), "fold_2d")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_unfold_into_a_transposed_output(dtype):
    """Columns written through a transposed view (column stride = rows)."""
    import torch

    import oracle
    from tensorrs_b200 import device
    x = rand([2, 3, 9, 11], dtype, 14)
    dx = contiguous(x)
    want = oracle.unfold_2d(dx.host_view(), (3, 3), (1, 1), (1, 1))
    rows, patch = want.shape
    out = empty([patch, rows], dtype).t()
    assert out.stride() == (1, rows)
    got = device.unfold_2d(dx.view, (3, 3), (1, 1), (1, 1), out)
    assert_bit_exact(to_host(got.contiguous()), want, "unfold into a transposed view")
    assert isinstance(got, torch.Tensor)


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_unfold_and_fold_with_padded_column_rows(dtype):
    """Columns whose rows are 4 entries longer than a window (row stride
    patch + 4, still 16-byte aligned): unfold writes only the window entries,
    fold reads them through the wider rows."""
    import oracle
    from tensorrs_b200 import device
    shape, k, s, p = [2, 8, 9, 10], (3, 3), (1, 1), (1, 1)
    x = rand(shape, dtype, 15)
    dx = contiguous(x)
    want = oracle.unfold_2d(dx.host_view(), k, s, p)
    rows, patch = want.shape
    wide = empty([rows, patch + 4], dtype)
    wide.fill_(7)
    device.unfold_2d(dx.view, k, s, p, wide[:, :patch])
    host = to_host(wide)
    assert_bit_exact(host[:, :patch], want, "unfold into padded rows")
    assert np.all(host[:, patch:] == 7)
    c = rand([rows, patch + 4], dtype, 16)
    dc = DevView(c, [rows, patch], [patch + 4, 1], 0)
    back = to_host(device.fold_2d(dc.view, k, s, p, empty(shape, dtype)))
    assert_bit_exact(back, oracle.fold_2d(dc.host_view(), shape, k, s, p), "fold from padded rows")


def test_unfold_of_a_strided_image_and_fold_errors():
    import oracle
    from tensorrs_b200 import abi, device
    base = rand([2, 3, 10, 12], np.float32, 11)
    # every other column of a [2, 3, 10, 12] image: a [2, 3, 10, 6] view
    dx = DevView(base, [2, 3, 10, 6], [360, 120, 12, 2], 1)
    want = oracle.unfold_2d(dx.host_view(), (3, 3), (1, 1), (1, 1))
    got = to_host(device.unfold_2d(dx.view, (3, 3), (1, 1), (1, 1), empty(want.shape, np.float32)))
    assert_bit_exact(got, want, "unfold of a strided view")
    with pytest.raises(abi.TrsError) as e:
        device.fold_2d(contiguous(np.ones([5, 9], np.float32)).view, (3, 3), (1, 1), (0, 0),
                       empty([1, 1, 4, 4], np.float32))
    assert "!!!fold_2d(): shape [5, 9] does not match an unfold of [1, 1, 4, 4]!!!" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.unfold_2d(contiguous(np.ones([1, 1, 2, 2], np.float32)).view, (3, 3), (1, 1), (0, 0),
                         empty([1, 9], np.float32))
    assert "kernel does not fit a 2x2 input padded by (0, 0)" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.unfold_2d(contiguous(np.ones([1, 2, 2], np.float32)).view, (1, 1), (1, 1), (0, 0),
                         empty([4, 1], np.float32))
    assert "!!!unfold_2d() expects [batch, channels, height, width], got [1, 2, 2]!!!" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.unfold_2d(contiguous(np.ones([1, 1, 2, 2], np.float32)).view, (1, 1), (0, 1), (0, 0),
                         empty([4, 1], np.float32))
    assert "!!!unfold_2d(): stride must be positive!!!" in e.value.message


def test_conv2d_as_unfold_then_matmul():
    """Conv2d::forward's data path (nn/conv2d.rs:217-241): unfold the input,
    multiply by the [C*kh*kw, out] weight, bit for bit against the same chain
    on the oracle."""
    import oracle
    from tensorrs_b200 import device
    x = rand([4, 8, 16, 16], np.float32, 12)
    w = rand([8 * 9, 32], np.float32, 13)
    dx, dw = contiguous(x), contiguous(w)
    cols_ref = oracle.unfold_2d(dx.host_view(), (3, 3), (1, 1), (1, 1))
    want = oracle.matmul(oracle.contiguous(cols_ref), dw.host_view())
    cols = device.unfold_2d(dx.view, (3, 3), (1, 1), (1, 1), empty(cols_ref.shape, np.float32))
    out = device.matmul(device.view_of(cols), dw.view, empty(want.shape, np.float32))
    assert_bit_exact(to_host(out), want, "conv2d as unfold + matmul")


def test_unfold_and_fold_at_the_benchmark_size():
    """unfold_2d / fold_2d of the measured configuration, X f32 [32, 64, 56, 56]
    ~N(0,1), 3x3 windows, stride 1, padding 1 (57.8 M column elements), bit
    for bit against the oracle."""
    import oracle
    from tensorrs_b200 import device
    shape = [32, 64, 56, 56]
    x = oracle.fill_normal(np.float32, int(np.prod(shape)), 7).reshape(shape)
    dx = contiguous(x)
    want = oracle.unfold_2d(dx.host_view(), (3, 3), (1, 1), (1, 1))
    cols = device.unfold_2d(dx.view, (3, 3), (1, 1), (1, 1), empty(want.shape, np.float32))
    assert_bit_exact(to_host(cols), want, "unfold_2d at the benchmark size")
    c = oracle.fill_normal(np.float32, want.size, 8).reshape(want.shape)
    dc = contiguous(c)
    back = to_host(device.fold_2d(dc.view, (3, 3), (1, 1), (1, 1), empty(shape, np.float32)))
    assert_bit_exact(back, oracle.fold_2d(dc.host_view(), shape, (3, 3), (1, 1), (1, 1)), "fold_2d at the benchmark size")
