"""Parity at the five benchmark configurations, at their full sizes, seeds and
distributions, through the C ABI against the oracle.

Inputs (the same streams bench.py times):
  1. A f32 [1024, 1024] ~U(-1,1) = seed-0 elements [0, 2^20), row bias b [1024]
     = seed-0 elements [2^20, 2^20 + 1024);
  2. A, B f32 [4096, 4096] ~N(0,1) = seed-1 elements [0, n^2) and [n^2, 2 n^2);
     B^T is the strided view (strides [1, 4096]) of B, never copied;
  3. X f32 [8192, 16384] ~N(0,1), seed 2;
  4. X f32 [64, 256, 56, 56] ~N(0,1) = seed-3 elements [0, N), upstream grad G
     = seed-3 elements [N, 2N); scale s [1,256,1,1] ~U(0.5,1.5) = seed-3
     uniforms [0, 256), bias b ~U(-0.1,0.1) = seed-3 uniforms [256, 512);
  5. A, B f32 [65536, 32768] ~U(-1,1) from seeds 4 and 5, c [32768] from seed 6
     (generated on the device; the device generator is bit-identical to the
     oracle's, tested in test_ew_gpu.py).

Tolerances: element-wise results and max/argmax bit-exact; sigmoid within
2 ulp; sums and means (f64 accumulation on the GPU, rounded once) within
1e-5 * sum|x| of the reference's sequential f32 fold and within
ulp(exact) + n * 2^-53 * sum|x| of the exact sum (checked as 2^-23 |exact| +
2^-40 sum|x| per output, as in test_reduce_gpu.py).

Config 3's axis-0 reductions and softmax at full size are in
test_reduce_col_gpu.py and test_softmax_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import contiguous, empty, to_host
from _util import assert_bit_exact, max_ulp, ulp_diff

pytestmark = pytest.mark.gpu


def check_sum(got, ref, x_abs_sum, exact):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape
    worst = float(np.max(np.abs(got - ref) - 1e-5 * np.asarray(x_abs_sum)))
    assert np.all(np.abs(got - ref) <= 1e-5 * np.asarray(x_abs_sum) + 1e-30), worst
    tol = np.abs(exact) * 2.0**-23 + 2.0**-40 * np.asarray(x_abs_sum) + 1e-300
    assert np.all(np.abs(got - exact) <= tol)


def _release():
    import torch
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# config 1: A + b, then sum over axis 1 and the full sum (seed 0)
# ---------------------------------------------------------------------------
def test_config1_bias_add_row_sums_and_sum():
    import oracle
    from tensorrs_b200 import abi, device
    n = 1024
    a = oracle.fill_uniform(np.float32, n * n, 0).reshape(n, n)
    b = oracle.fill_uniform(np.float32, n, 0, first=n * n)
    da, db = contiguous(a), contiguous(b)
    y = empty([n, n], np.float32)
    device.binary("add", da.view, db.view, y)
    want = oracle.binary("add", da.host_view(), db.host_view())
    got_y = to_host(y)
    assert_bit_exact(got_y, want, "A + b")
    dy = contiguous(got_y)
    rows = to_host(device.sum_axis(dy.view, 1, False, empty([n], np.float32)))
    ref_rows = oracle.sum_axis(dy.host_view(), 1, False)
    yd = want.astype(np.float64)
    check_sum(rows, ref_rows, np.abs(yd).sum(axis=1), yd.sum(axis=1))
    s = to_host(device.sum_all(dy.view, empty([1], np.float32)))
    exact, sabs = oracle.sum_f64(dy.host_view())
    check_sum(s, [oracle.sum_all(dy.host_view())], [sabs], [exact])
    # A + b and sum(A + b) in one fused call
    y2 = empty([n, n], np.float32)
    s2 = empty([1], np.float32)
    device.elementwise(abi.program(2, abi.ADD), [da.view, db.view], y2, s2)
    assert_bit_exact(to_host(y2), want, "A + b (fused with its sum)")
    check_sum(to_host(s2), [oracle.sum_all(dy.host_view())], [sabs], [exact])
    # the whole chain (A + b, its row sums, its sum) in one pass
    y3, r3, s3 = empty([n, n], np.float32), empty([n], np.float32), empty([1], np.float32)
    device.elementwise_row_sums(abi.program(2, abi.ADD), [da.view, db.view], y3, r3, s3)
    assert_bit_exact(to_host(y3), want, "A + b (one pass with its sums)")
    check_sum(to_host(r3), ref_rows, np.abs(yd).sum(axis=1), yd.sum(axis=1))
    check_sum(to_host(s3), [oracle.sum_all(dy.host_view())], [sabs], [exact])


# ---------------------------------------------------------------------------
# config 2: C = A & B^T with B^T a strided view, then sigmoid (seed 1)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def config2():
    import oracle
    n = 4096
    a = oracle.fill_normal(np.float32, n * n, 1).reshape(n, n)
    b = oracle.fill_normal(np.float32, n * n, 1, first=n * n).reshape(n, n)
    return n, a, b


def test_config2_mul_by_transposed_view_bit_exact(config2):
    import oracle
    from tensorrs_b200 import device
    n, a, b = config2
    da = contiguous(a)
    db = contiguous(b)
    db.shape, db.strides = [n, n], [1, n]  # B^T: no copy
    got = to_host(device.binary("mul", da.view, db.view, empty([n, n], np.float32)))
    want = oracle.binary("mul", da.host_view(), db.host_view())
    assert_bit_exact(got, want, "A & B^T")
    _release()


def test_config2_sigmoid_fused_and_standalone_within_two_ulp(config2):
    import oracle
    from tensorrs_b200 import abi, device
    n, a, b = config2
    da = contiguous(a)
    db = contiguous(b)
    db.shape, db.strides = [n, n], [1, n]
    fused = empty([n, n], np.float32)
    device.elementwise(abi.program(2, abi.MUL, epilogue="sigmoid"), [da.view, db.view], fused)
    prod = oracle.binary("mul", da.host_view(), db.host_view())
    want = oracle.unary("sigmoid", oracle.contiguous(prod))
    got = to_host(fused)
    u = max_ulp(got, want)
    same = float((ulp_diff(got, want) == 0).mean())
    print(f"sigmoid(A & B^T) fused: max {u} ulp, {same:.4%} bit-identical")
    assert u <= 2
    # the standalone map over the materialised product
    dp = contiguous(prod)
    alone = to_host(device.unary("sigmoid", dp.view, empty([n, n], np.float32)))
    u2 = max_ulp(alone, want)
    print(f"sigmoid standalone: max {u2} ulp, {float((ulp_diff(alone, want) == 0).mean()):.4%} bit-identical")
    assert u2 <= 2
    _release()


# ---------------------------------------------------------------------------
# config 3: reductions over axis 1 of X [8192, 16384] (seed 2)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def config3():
    import oracle
    x = oracle.fill_normal(np.float32, 8192 * 16384, 2).reshape(8192, 16384)
    xd = x.astype(np.float64)
    return x, xd.sum(axis=1), np.abs(xd).sum(axis=1)


def test_config3_sum_and_mean_over_axis1(config3):
    import oracle
    from tensorrs_b200 import device
    x, exact, sabs = config3
    dx = contiguous(x)
    got = to_host(device.sum_axis(dx.view, 1, False, empty([8192], np.float32)))
    check_sum(got, oracle.sum_axis(dx.host_view(), 1, False), sabs, exact)
    kd = to_host(device.sum_axis(dx.view, 1, True, empty([8192, 1], np.float32)))
    assert_bit_exact(kd.reshape(-1), got, "keepdim sum")
    mean = to_host(device.mean_axis(dx.view, 1, False, empty([8192], np.float32)))
    ref_mean = oracle.mean_axis(dx.host_view(), 1, False)
    # the mean is the f32 sum divided by n with one IEEE division
    assert_bit_exact(mean, (got / np.float32(16384)).astype(np.float32), "mean = sum / n")
    check_sum(mean, ref_mean, sabs / 16384, exact / 16384)
    _release()


def test_config3_max_and_argmax_over_axis1(config3):
    import oracle
    from tensorrs_b200 import device
    x, _, _ = config3
    dx = contiguous(x)
    vals = to_host(device.max_axis(dx.view, 1, empty([8192], np.float32)))
    idx = to_host(device.argmax_axis(dx.view, 1, empty([8192], np.int64)))
    rv, ri = oracle.max_argmax_axis(dx.host_view(), 1)
    assert_bit_exact(vals, rv, "max_axis(1)")
    assert_bit_exact(idx, ri, "argmax_axis(1)")
    _release()


def test_config3_mean_over_axis0(config3):
    import oracle
    from tensorrs_b200 import device
    x, _, _ = config3
    dx = contiguous(x)
    got = to_host(device.mean_axis(dx.view, 0, False, empty([16384], np.float32)))
    ref = oracle.mean_axis(dx.host_view(), 0, False)
    xd = x.astype(np.float64)
    check_sum(got, ref, np.abs(xd).sum(axis=0) / 8192, xd.sum(axis=0) / 8192)
    _release()


# ---------------------------------------------------------------------------
# config 4: relu(X & s + b) forward, scale and bias gradients (seed 3)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def config4():
    import oracle
    shape = [64, 256, 56, 56]
    n = int(np.prod(shape))
    x = oracle.fill_normal(np.float32, n, 3).reshape(shape)
    g = oracle.fill_normal(np.float32, n, 3, first=n).reshape(shape)
    s = oracle.fill_uniform(np.float32, 256, 3, 0.5, 1.5).reshape(1, 256, 1, 1)
    b = oracle.fill_uniform(np.float32, 256, 3, -0.1, 0.1, first=256).reshape(1, 256, 1, 1)
    return shape, x, g, s, b


def test_config4_affine_relu_forward_bit_exact(config4):
    import oracle
    from tensorrs_b200 import abi, device
    shape, x, _, s, b = config4
    dx, ds, db = contiguous(x), contiguous(s), contiguous(b)
    y = empty(shape, np.float32)
    device.elementwise(abi.program(3, abi.MUL, abi.ADD, "relu"), [dx.view, ds.view, db.view], y)
    want = oracle.program(3, "mul", "add", "relu", [dx.host_view(), ds.host_view(), db.host_view()])
    assert_bit_exact(to_host(y), want, "relu(X & s + b)")
    _release()


def test_config4_scale_and_bias_gradients(config4):
    """The reference's chain (autodiff/core.rs:173-227 with relu.rs:32-42):
    bias grad = reduce_to_shape(g & mask), scale grad = reduce_to_shape((g &
    mask) & X), each reduced pass by pass (base.rs:1651-1686)."""
    import oracle
    from tensorrs_b200 import device
    shape, x, g, s, b = config4
    dx, dg, ds, db = contiguous(x), contiguous(g), contiguous(s), contiguous(b)
    z = oracle.program(3, "mul", "add", "none", [dx.host_view(), ds.host_view(), db.host_view()])
    mask = (z > 0).astype(np.float32)
    del z
    gm = oracle.binary("mul", dg.host_view(), oracle.contiguous(mask))
    del mask
    gmx = oracle.binary("mul", oracle.contiguous(gm), dx.host_view())
    t = [1, 256, 1, 1]
    gs, gb = empty(t, np.float32), empty(t, np.float32)
    device.affine_relu_backward(dg.view, dx.view, ds.view, db.view, gs, gb)
    for got, prod, what in [(to_host(gs), gmx, "scale grad"), (to_host(gb), gm, "bias grad")]:
        ref = oracle.reduce_broadcast_grad(oracle.contiguous(prod), t)
        pd = prod.astype(np.float64)
        exact = pd.sum(axis=(0, 2, 3), keepdims=True)
        sabs = np.abs(pd).sum(axis=(0, 2, 3), keepdims=True)
        check_sum(got, ref, sabs, exact)
    _release()


def test_config4_reduce_broadcast_grad(config4):
    import oracle
    from tensorrs_b200 import abi, device
    shape, _, g, _, _ = config4
    dg = contiguous(g)
    t = [1, 256, 1, 1]
    out = empty(t, np.float32)
    assert device.reduce_broadcast_grad(dg.view, t, out) == abi.OK
    ref = oracle.reduce_broadcast_grad(dg.host_view(), t)
    gd = g.astype(np.float64)
    check_sum(to_host(out), ref, np.abs(gd).sum(axis=(0, 2, 3), keepdims=True),
              gd.sum(axis=(0, 2, 3), keepdims=True))
    _release()


# ---------------------------------------------------------------------------
# config 5: Y = A & B + c and sum(Y) on one GPU at full size (seeds 4, 5, 6)
# ---------------------------------------------------------------------------
def test_config5_fused_multiply_add_and_sum_full_size():
    """Every element of Y is checked through per-row checksums of its bit
    patterns (a single differing element changes its row's), a spread of rows
    bit for bit, and sum(Y) against the reference's sequential f32 fold and
    the exact sum -- the oracle regenerates the 2^31 elements from the seeds
    instead of holding them."""
    import torch

    import oracle
    from tensorrs_b200 import abi, device
    rows, cols = 65536, 32768
    f32 = torch.float32
    A = device.fill_uniform(torch.empty((rows, cols), dtype=f32, device="cuda"), 4)
    B = device.fill_uniform(torch.empty((rows, cols), dtype=f32, device="cuda"), 5)
    c = device.fill_uniform(torch.empty((cols,), dtype=f32, device="cuda"), 6)
    Y = torch.empty((rows, cols), dtype=f32, device="cuda")
    S = torch.empty((1,), dtype=f32, device="cuda")
    device.elementwise(abi.program(3, abi.MUL, abi.ADD), [device.view_of(A), device.view_of(B),
                                                          device.view_of(c)], Y, S)
    del A, B
    torch.cuda.synchronize()
    s_gpu = float(S.cpu()[0])
    # per-row checksums on the device, in slabs of 4096 rows
    bits = np.empty(rows, dtype=np.int64)
    for r0 in range(0, rows, 4096):
        bits[r0:r0 + 4096] = Y[r0:r0 + 4096].view(torch.int32).to(torch.int64).sum(dim=1).cpu().numpy()
    spot = [0, 1, 4095, 4096, 32767, 32768, 54321, 65535]
    got_rows = Y[spot].cpu().numpy()
    del Y
    _release()
    fold, exact, sabs, ref_bits = oracle.fma_sum_stream(rows, cols, 4, 5, 6, row_bits=True)
    bad = np.flatnonzero(bits != ref_bits)
    assert bad.size == 0, f"{bad.size} rows differ in their bit checksum, e.g. {bad[:5]}"
    cc = oracle.fill_uniform(np.float32, cols, 6)
    for k, r in enumerate(spot):
        ar = oracle.fill_uniform(np.float32, cols, 4, first=r * cols)
        br = oracle.fill_uniform(np.float32, cols, 5, first=r * cols)
        want = oracle.program(3, "mul", "add", "none", [oracle.contiguous(ar), oracle.contiguous(br),
                                                        oracle.contiguous(cc)])
        assert_bit_exact(got_rows[k], want, f"row {r} of Y")
    n = rows * cols
    print(f"sum(Y): gpu {s_gpu!r}, reference fold {float(fold)!r}, exact {exact!r}, sum|y| {sabs:.6g}; "
          f"|gpu - fold| / sum|y| = {abs(s_gpu - float(fold)) / sabs:.3g}, "
          f"|gpu - exact| = {abs(s_gpu - exact):.3g}")
    assert abs(s_gpu - float(fold)) <= 1e-5 * sabs
    ulp = float(np.spacing(np.float32(abs(exact))))
    assert abs(s_gpu - exact) <= ulp + n * 2.0**-53 * sabs
