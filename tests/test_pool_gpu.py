"""The pooling layers on the GPU through the C ABI, bit-exact against the
oracle's restatement of the reference (reshape -> unfold_2d -> max_axis, or
sum_axis / (kh * kw); max_axis's backward -> fold_2d):

* the forward kernels: the TMA row-box kernel (rows of a multiple of 16 bytes
  and at most 256 elements, any window: overlapping, gapped, planes split into
  several boxes of rows; f32 3x3 and 2x2 windows at stride 2 two outputs per
  thread), the 16-byte strip kernel (kw == stride_w dividing 16 bytes, its
  ragged row ends), the shared-memory tile kernel (wider rows) and the general
  one (other views, strided outputs);
* NaN as a window's first element and elsewhere, +-inf, -0 / +0 ties;
* MaxPool2d's gradient through the TMA row-box kernel (f32 2x2 windows at
  stride 2 tiling the image), the strip, tile and general kernels with
  ties, overlapping windows (a pixel collecting from several windows, blocks
  taking windows from the block above), uncovered edge pixels, and the
  accumulation onto a held gradient;
* the config-4 activation shape [64, 256, 56, 56] at full size;
* the errors the reference panics with, aliasing and empty tensors.
"""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact

pytestmark = pytest.mark.gpu


def _special(x):
    x = x.copy()
    flat = x.reshape(-1)
    flat[0] = np.nan
    if flat.size > 40:
        flat[37] = np.nan
        flat[11] = np.inf
        flat[12] = -np.inf
        flat[20:24] = [-0.0, 0.0, 0.0, -0.0]
    return x


def _ties(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    vals = np.array([-2.0, -1.0, -0.0, 0.0, 0.5, 1.0, 3.0], dtype)
    return vals[rng.integers(0, vals.size, size=shape)]


def _fwd(kind, dv, kernel, stride, dtype):
    from tensorrs_b200 import device
    n, c, h, w = dv.shape
    oh, ow = device.pooled_size((h, w), kernel, stride)
    fn = device.max_pool2d if kind == "max" else device.avg_pool2d
    return to_host(fn(dv.view, kernel, empty([n, c, oh, ow], dtype), stride))


FWD = [
    # (shape, kernel, stride): strips (f32 kw 1/2/4, f64 kw 1/2) with and
    # without ragged row ends, then the general kernel
    ([2, 3, 8, 8], (2, 2), (2, 2)),
    ([2, 3, 9, 10], (2, 2), (2, 2)),     # f64 strips; f32 rows not 16-byte aligned
    ([3, 2, 7, 16], (3, 4), (2, 4)),     # f32 strips of one window
    ([2, 5, 6, 12], (2, 1), (3, 1)),     # strips of 4 (f32) / 2 (f64) one-column windows
    ([4, 16, 56, 56], (2, 2), (2, 2)),
    ([2, 3, 9, 9], (3, 3), (2, 2)),
    ([2, 3, 7, 10], (2, 2), (1, 1)),
    ([1, 2, 5, 11], (1, 2), (1, 1)),
    ([2, 2, 11, 7], (3, 1), (2, 3)),
    ([1, 3, 32, 33], (5, 3), (3, 2)),
    # shared-memory tiles: rows of a multiple of 16 bytes, any window
    ([2, 3, 9, 12], (3, 3), (2, 2)),
    ([2, 4, 56, 56], (3, 3), (2, 2)),
    ([1, 2, 5, 8], (1, 2), (1, 1)),
    ([2, 2, 11, 8], (3, 1), (2, 3)),
    ([1, 3, 32, 36], (5, 3), (3, 2)),
    ([1, 2, 64, 1024], (3, 3), (2, 2)),   # several blocks of rows per plane
    ([1, 2, 600, 40], (3, 3), (2, 2)),    # several TMA boxes of rows per plane
    ([1, 1, 4, 8192], (1, 3), (1, 2)),    # rows too wide for a tile: the general kernel
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("kind", ["max", "avg"])
@pytest.mark.parametrize("case", FWD, ids=lambda c: f"{c[0]}-k{c[1]}-s{c[2]}")
def test_pool_forward_bit_exact(case, kind, dtype):
    import oracle
    shape, kernel, stride = case
    x = _special(np.random.default_rng(sum(shape)).standard_normal(shape).astype(dtype))
    dv = contiguous(x)
    got = _fwd(kind, dv, kernel, stride, dtype)
    assert_bit_exact(got, oracle.pool2d(kind, dv.host_view(), kernel, stride), f"{kind} {case}")


@pytest.mark.parametrize("kind", ["max", "avg"])
def test_pool_forward_ties_and_signed_zeros(kind):
    import oracle
    x = _ties([3, 4, 12, 16], np.float32, 1)
    dv = contiguous(x)
    # 2x2 / 3x3 at stride 2: two outputs per thread (3x3: an odd OW, the last thread's second one skipped)
    for kernel, stride in [((2, 2), (2, 2)), ((3, 3), (2, 2)), ((3, 3), (1, 1)), ((2, 4), (2, 4))]:
        got = _fwd(kind, dv, kernel, stride, np.float32)
        want = oracle.pool2d(kind, dv.host_view(), kernel, stride)
        assert_bit_exact(got, want, f"{kind} ties {kernel}")


@pytest.mark.parametrize("kind", ["max", "avg"])
def test_pool_forward_strided_and_misaligned_views(kind):
    """An H/W-transposed input, a channel slice, an offset of one element
    (16-byte alignment lost: the general kernel), rows narrower than their
    pitch (the strip kernel's ragged row end), and a strided output."""
    import oracle
    from tensorrs_b200 import device
    rng = np.random.default_rng(8)
    st = rng.standard_normal(2 * 6 * 12 * 16 + 1).astype(np.float32)
    views = [
        ([2, 6, 16, 12], [1152, 192, 1, 16], 0),      # H and W swapped
        ([2, 3, 12, 16], [1152, 384, 16, 1], 192),    # every other channel, from channel 1
        ([2, 6, 12, 16], [1152, 192, 16, 1], 1),      # offset 1: unaligned rows
        ([2, 6, 12, 14], [1152, 192, 16, 1], 0),      # rows of 14 in a pitch of 16: a ragged last strip
    ]
    for shape, strides, off in views:
        dv = DevView(st, shape, strides, off)
        want = oracle.pool2d(kind, dv.host_view(), (2, 2), (2, 2))
        assert_bit_exact(_fwd(kind, dv, (2, 2), (2, 2), np.float32), want, f"{kind} view {strides} +{off}")
    # a strided output: every other element of a wider buffer
    dv = contiguous(st[:2 * 6 * 12 * 16].reshape(2, 6, 12, 16))
    big = empty([2, 6, 6, 16], np.float32)
    big.zero_()
    out_view = device.view_of(big, [2, 6, 6, 8], [576, 96, 16, 2], 0)
    fn = "trs_max_pool2d" if kind == "max" else "trs_avg_pool2d"
    import ctypes
    device._call(fn, ctypes.byref(dv.view), 2, 2, 2, 2, ctypes.byref(out_view), device.stream_handle())
    got = to_host(big)[:, :, :, 0::2]
    assert_bit_exact(got, oracle.pool2d(kind, dv.host_view(), (2, 2), (2, 2)), "strided output")
    assert not to_host(big)[:, :, :, 1::2].any()


def test_pool_forward_full_config4_size():
    """MaxPool2d and AvgPool2d 2x2 over the [64, 256, 56, 56] activation."""
    import oracle
    x = np.random.default_rng(3).standard_normal((64, 256, 56, 56)).astype(np.float32)
    dv = contiguous(x)
    for kind in ("max", "avg"):
        got = _fwd(kind, dv, (2, 2), (2, 2), np.float32)
        assert_bit_exact(got, oracle.pool2d(kind, dv.host_view(), (2, 2), (2, 2)), kind)


BWD = [
    ([2, 3, 8, 8], (2, 2), (2, 2)),
    ([2, 3, 9, 11], (2, 2), (2, 2)),     # an uncovered last row and column
    ([2, 3, 9, 9], (3, 3), (2, 2)),      # overlapping windows
    ([2, 2, 7, 10], (2, 2), (1, 1)),
    ([1, 2, 4, 9], (1, 2), (1, 1)),
    ([2, 2, 11, 7], (2, 1), (3, 3)),     # gaps between windows
    # shared-memory tiles
    ([2, 3, 9, 12], (3, 3), (2, 2)),
    ([2, 2, 7, 12], (2, 2), (1, 1)),
    ([1, 2, 4, 8], (1, 2), (1, 1)),
    ([2, 2, 11, 8], (2, 1), (3, 3)),
    ([1, 2, 40, 1024], (3, 3), (2, 2)),  # blocks that take windows from the block above
    ([1, 2, 600, 16], (2, 2), (2, 2)),   # several TMA row blocks per plane
    ([1, 2, 13, 16], (5, 2), (1, 2)),    # windows five rows high at stride 1
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("case", BWD, ids=lambda c: f"{c[0]}-k{c[1]}-s{c[2]}")
def test_max_pool_backward_bit_exact(case, dtype):
    import oracle
    from tensorrs_b200 import device
    shape, kernel, stride = case
    x = _ties(shape, dtype, sum(shape))
    x.reshape(-1)[5] = np.nan
    n, c, h, w = shape
    oh, ow = device.pooled_size((h, w), kernel, stride)
    g = np.random.default_rng(4).standard_normal((n, c, oh, ow)).astype(dtype)
    g.reshape(-1)[0] = -0.0
    dx, dg = contiguous(x), contiguous(g)
    got = to_host(device.max_pool2d_backward(dx.view, dg.view, kernel, empty(shape, dtype), stride))
    assert_bit_exact(got, oracle.max_pool2d_backward(dx.host_view(), dg.host_view(), kernel, stride), "grad")
    # accumulated onto a held gradient with signed zeros in it
    cur = np.random.default_rng(5).standard_normal(shape).astype(dtype)
    cur.reshape(-1)[:8] = -0.0
    import torch
    held = torch.from_numpy(cur.copy()).cuda()
    got = to_host(device.max_pool2d_backward(dx.view, dg.view, kernel, held, stride, accumulate=True))
    want = oracle.max_pool2d_backward(dx.host_view(), dg.host_view(), kernel, stride, current=cur)
    assert_bit_exact(got, want, "accumulated grad")


def test_max_pool_backward_full_config4_size():
    import oracle
    from tensorrs_b200 import device
    x = np.random.default_rng(6).standard_normal((64, 256, 56, 56)).astype(np.float32)
    g = np.random.default_rng(7).standard_normal((64, 256, 28, 28)).astype(np.float32)
    dx, dg = contiguous(x), contiguous(g)
    got = to_host(device.max_pool2d_backward(dx.view, dg.view, (2, 2), empty(x.shape, np.float32)))
    assert_bit_exact(got, oracle.max_pool2d_backward(dx.host_view(), dg.host_view(), (2, 2)), "grad")


def test_pool_errors_and_empty():
    import torch

    from tensorrs_b200 import abi, device
    x = contiguous(np.ones((1, 2, 4, 4), np.float32))

    def status(fn):
        with pytest.raises(abi.TrsError) as e:
            fn()
        return e.value.status

    out = empty([1, 2, 2, 2], np.float32)
    assert status(lambda: device.max_pool2d(contiguous(np.ones((4, 4), np.float32)).view, (2, 2), out)) == abi.ERR_SHAPE
    assert status(lambda: device.max_pool2d(x.view, (2, 2), out, (0, 2))) == abi.ERR_ARG
    assert status(lambda: device.max_pool2d(x.view, (5, 2), out)) == abi.ERR_SHAPE
    assert status(lambda: device.max_pool2d(x.view, (2, 2), empty([1, 2, 2, 3], np.float32))) == abi.ERR_SHAPE
    assert status(lambda: device.max_pool2d(x.view, (0, 2), empty([1, 2, 5, 2], np.float32), (1, 2))) \
        == abi.ERR_EMPTY_AXIS
    assert status(lambda: device.max_pool2d(x.view, (2, 2), empty([1, 2, 2, 2], np.float64))) == abi.ERR_DTYPE
    xi = contiguous(np.ones((1, 2, 4, 4), np.int32))
    assert status(lambda: device.max_pool2d(xi.view, (2, 2), empty([1, 2, 2, 2], np.int32))) == abi.ERR_DTYPE
    # the output inside the input's storage
    assert status(lambda: device.max_pool2d(x.view, (2, 2), x.t[:8].view(1, 2, 2, 2))) == abi.ERR_ALIAS
    g = contiguous(np.ones((1, 2, 2, 2), np.float32))
    assert status(lambda: device.max_pool2d_backward(x.view, g.view, (2, 2), x.t.view(1, 2, 4, 4))) == abi.ERR_ALIAS
    # an empty window averages to 0 / 0
    avg = to_host(device.avg_pool2d(x.view, (0, 2), empty([1, 2, 5, 2], np.float32), (1, 2)))
    assert np.isnan(avg).all()
    # empty batch: nothing to do
    e = contiguous(np.ones((0, 2, 4, 4), np.float32))
    device.max_pool2d(e.view, (2, 2), empty([0, 2, 2, 2], np.float32))
    device.max_pool2d_backward(e.view, contiguous(np.ones((0, 2, 2, 2), np.float32)).view, (2, 2),
                               empty([0, 2, 4, 4], np.float32))
    torch.cuda.synchronize()
