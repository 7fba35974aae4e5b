"""The oracle's pooling (MaxPool2d / AvgPool2d forward, MaxPool2d's gradient)
pinned beyond the reference's known answers against an independent numpy
restatement: windows read straight from the input by slicing (no unfold), a
strict `>` scan from the window's first element, sums added one numpy scalar
operation at a time in window order from 0, and the gradient scattered window
by window in (oh, ow) order.  Also the host-side shape rule (pooled_size) and
the errors the reference panics with."""
from __future__ import annotations

import numpy as np
import pytest


def _windows(x, kh, kw, sh, sw):
    n, c, h, w = x.shape
    oh, ow = (h - kh) // sh + 1, (w - kw) // sw + 1
    for b in range(n):
        for ch in range(c):
            for i in range(oh):
                for j in range(ow):
                    yield (b, ch, i, j), x[b, ch, i * sh:i * sh + kh, j * sw:j * sw + kw].reshape(-1)


def _np_pool(kind, x, kh, kw, sh, sw):
    n, c, h, w = x.shape
    T = x.dtype.type
    out = np.empty((n, c, (h - kh) // sh + 1, (w - kw) // sw + 1), x.dtype)
    for at, win in _windows(x, kh, kw, sh, sw):
        if kind == "max":
            best = win[0]
            for v in win[1:]:
                if v > best:
                    best = v
            out[at] = best
        else:
            acc = T(0)
            for v in win:
                acc = T(acc + v)
            out[at] = T(acc / T(kh * kw))
    return out


def _np_max_backward(x, g, kh, kw, sh, sw):
    T = x.dtype.type
    gx = np.zeros_like(x)
    for (b, ch, i, j), win in _windows(x, kh, kw, sh, sw):
        best, at = win[0], 0
        for k in range(1, win.size):
            if win[k] > best:
                best, at = win[k], k
        u, v = divmod(at, kw)
        y, xx = i * sh + u, j * sw + v
        gx[b, ch, y, xx] = T(gx[b, ch, y, xx] + g[b, ch, i, j])
    return gx


def _quantised(shape, dtype, seed):
    """Values from a small set, so windows hold ties (+0 and -0 among them)."""
    rng = np.random.default_rng(seed)
    vals = np.array([-2.0, -1.0, -0.0, 0.0, 0.5, 1.0, 3.0], dtype)
    return vals[rng.integers(0, vals.size, size=shape)]


GEOMS = [((2, 2), (2, 2)), ((3, 3), (2, 2)), ((2, 2), (1, 1)), ((1, 2), (1, 1)), ((3, 1), (2, 3)), ((2, 3), (3, 1))]


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("geom", GEOMS, ids=str)
def test_oracle_pool_forward_matches_numpy(orc, geom, dtype):
    (kh, kw), (sh, sw) = geom
    rng = np.random.default_rng(kh * 7 + kw)
    x = rng.standard_normal((2, 3, 9, 11)).astype(dtype)
    x[0, 0, 0, 0] = np.nan          # a NaN first element of its window stays
    x[1, 2, 4, 5] = np.nan          # elsewhere it never wins a strict `>`
    x[0, 1, :3, :3] = -np.inf
    for kind in ("max", "avg"):
        got = orc.pool2d(kind, orc.contiguous(x), (kh, kw), (sh, sw))
        want = _np_pool(kind, x, kh, kw, sh, sw)
        assert got.shape == want.shape
        np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("geom", GEOMS, ids=str)
def test_oracle_max_pool_backward_matches_numpy(orc, geom):
    (kh, kw), (sh, sw) = geom
    x = _quantised((2, 3, 8, 10), np.float32, kh + 10 * kw)
    oh, ow = (8 - kh) // sh + 1, (10 - kw) // sw + 1
    g = np.random.default_rng(5).standard_normal((2, 3, oh, ow)).astype(np.float32)
    g[0, 0, 0, 0] = -0.0
    got = orc.max_pool2d_backward(orc.contiguous(x), orc.contiguous(g), (kh, kw), (sh, sw))
    want = _np_max_backward(x, g, kh, kw, sh, sw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    cur = np.random.default_rng(6).standard_normal(x.shape).astype(np.float32)
    got = orc.max_pool2d_backward(orc.contiguous(x), orc.contiguous(g), (kh, kw), (sh, sw), current=cur)
    np.testing.assert_array_equal(got, cur + want)


def test_oracle_pool_reads_strided_views(orc):
    rng = np.random.default_rng(3)
    st = rng.standard_normal(2 * 3 * 10 * 12).astype(np.float32)
    # [N, C, H, W] = [2, 3, 12, 10] as the H/W transpose of a [2, 3, 10, 12] storage
    v = orc.HostView(st, [2, 3, 12, 10], [360, 120, 1, 12], 0)
    xt = np.ascontiguousarray(st.reshape(2, 3, 10, 12).transpose(0, 1, 3, 2))
    for kind in ("max", "avg"):
        np.testing.assert_array_equal(orc.pool2d(kind, v, (3, 2), (2, 2)), _np_pool(kind, xt, 3, 2, 2, 2))


def test_oracle_pool_errors(orc):
    x = orc.contiguous(np.zeros((1, 1, 4, 4), np.float32))
    with pytest.raises(RuntimeError):
        orc.pool2d("max", orc.contiguous(np.zeros((4, 4), np.float32)), (2, 2))
    with pytest.raises(RuntimeError):
        orc.pool2d("max", x, (2, 2), (0, 1))
    with pytest.raises(RuntimeError):
        orc.pool2d("max", x, (5, 2))
    with pytest.raises(RuntimeError):
        orc.pool2d("max", x, (0, 2), (1, 2))    # max_axis over an empty axis
    avg = orc.pool2d("avg", x, (0, 2), (1, 2))  # sum of nothing, divided by 0
    assert avg.shape == (1, 1, 5, 2) and np.isnan(avg).all()


def test_pooled_size_matches_the_reference_doctests():
    from tensorrs_b200.device import pooled_size
    assert pooled_size((32, 32), (2, 2), (2, 2)) == (16, 16)   # nn/pool.rs:85-90
    assert pooled_size((9, 9), (3, 3), (2, 2)) == (4, 4)       # nn/pool.rs:102-107
    assert pooled_size((8, 8), (3, 3), (2, 2)) == (3, 3)       # nn/pool.rs:276-278
    with pytest.raises(ValueError):
        pooled_size((4, 4), (2, 2), (0, 2))
