"""trs_matmul_tf32x3: Tensor::matmul (linalg/tensor/base.rs:896-1013) for f32
on the tensor cores (tcgen05, split TF32), through the C ABI.

Not bit-identical by design (the tensor cores add the products in their own
order and precision): every output is held to
    |gpu - ref| <= 1e-5 * sum_k |a_ik b_kj|
against the reference's sequential f32 chain (the oracle), and, on these
shapes and seeds, to
    |gpu - exact| <= 2^-18 * sum_k |a_ik b_kj|
against the exact product (f64) -- a regression bound, not a worst case: the
split keeps products to about 2^-21, but an f32 accumulation of K terms can
err by up to (K - 1) 2^-24 sum|ab| (random signs keep it near sqrt(K) 2^-24;
the benchmark-size test below uses the worst case).  Shapes cover the padding of every tile edge (M, N not multiples of
128, K not a multiple of 32), batches with broadcasting, transposed and
offset views, K = 1 and K = 0."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host

pytestmark = pytest.mark.gpu


def rand(shape, seed):
    return np.random.default_rng(seed).standard_normal(size=shape).astype(np.float32)


def check(da: DevView, db: DevView):
    import oracle
    from tensorrs_b200 import device
    out = empty(device.matmul_shape(da.view, db.view), np.float32)
    got = to_host(device.matmul_tf32x3(da.view, db.view, out)).astype(np.float64)
    ref = oracle.matmul(da.host_view(), db.host_view()).astype(np.float64)
    a = np.array(oracle.unary("none", da.host_view()), np.float64)
    b = np.array(oracle.unary("none", db.host_view()), np.float64)
    exact = np.matmul(a, b)
    mag = np.matmul(np.abs(a), np.abs(b))
    assert got.shape == ref.shape
    worst = float(np.max(np.abs(got - ref) / np.maximum(mag, 1e-300))) if got.size else 0.0
    assert np.all(np.abs(got - ref) <= 1e-5 * mag + 1e-30), worst
    assert np.all(np.abs(got - exact) <= 2.0**-18 * mag + 1e-30)
    return worst


SHAPES = [
    ([128, 32], [32, 128]), ([256, 256], [256, 256]), ([129, 77], [77, 300]), ([1, 5], [5, 1]),
    ([300, 1], [1, 200]), ([2, 1, 70, 40], [3, 40, 50]), ([4, 64, 96], [96, 33]), ([1000, 513], [513, 257]),
]


@pytest.mark.parametrize("sa,sb", SHAPES, ids=lambda v: str(v))
def test_tf32x3_within_the_sum_tolerance(sa, sb):
    worst = check(contiguous(rand(sa, sum(sa))), contiguous(rand(sb, sum(sb) + 1)))
    print(f"{sa} x {sb}: worst |gpu - ref| / sum|ab| = {worst:.2e}")


def test_tf32x3_through_views_and_long_k():
    m, k, n = 200, 1500, 150
    a_t = rand([k, m], 3)
    b_t = rand([n, k], 4)
    check(DevView(a_t, [m, k], [1, m], 0), DevView(b_t, [k, n], [1, k], 0))  # A^T x B^T
    store = rand([m * (k + 3) + 7], 5)
    check(DevView(store, [m, k], [k + 3, 1], 7), contiguous(rand([k, n], 6)))
    check(contiguous(rand([512, 4096], 8)), contiguous(rand([4096, 384], 9)))


def test_tf32x3_empty_depth_gives_zeros_and_errors():
    from tensorrs_b200 import abi, device
    out = empty([3, 4], np.float32)
    got = to_host(device.matmul_tf32x3(contiguous(np.ones([3, 0], np.float32)).view,
                                       contiguous(np.ones([0, 4], np.float32)).view, out))
    assert np.array_equal(got, np.zeros([3, 4], np.float32)) and not np.signbit(got).any()
    with pytest.raises(abi.TrsError) as e:
        device.matmul_tf32x3(contiguous(np.ones([2, 3], np.float32)).view,
                             contiguous(np.ones([2, 3], np.float32)).view, empty([2, 3], np.float32))
    assert "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])" in e.value.message
    with pytest.raises(abi.TrsError) as e:
        device.matmul_tf32x3(contiguous(np.ones([2, 3], np.int32)).view,
                             contiguous(np.ones([3, 2], np.int32)).view, empty([2, 2], np.int32))
    assert e.value.status == abi.ERR_DTYPE


def test_tf32x3_no_kernel_gave_up_waiting():
    import ctypes

    from tensorrs_b200 import abi
    code = ctypes.c_int32(-1)
    abi.check(abi.load().trs_async_error(ctypes.byref(code)))
    assert code.value == 0


def test_tf32x3_non_finite_inputs_follow_the_reference():
    """An infinity or NaN among the inputs: a split product inf * (a zero lo
    part) would turn an infinite result into NaN, so such calls take the
    reference's exact chain and match the oracle bit for bit -- here against
    partners that are exact TF32 values (small integers), whose lo parts are 0."""
    import oracle
    from _util import assert_bit_exact
    from tensorrs_b200 import device
    rng = np.random.default_rng(41)
    a = rng.integers(-4, 5, size=[130, 40]).astype(np.float32)
    b = rng.integers(-4, 5, size=[40, 140]).astype(np.float32)
    a[3, 5] = np.inf
    a[7, 1] = np.nan
    b[2, 9] = -np.inf
    da, db = contiguous(a), contiguous(b)
    got = to_host(device.matmul_tf32x3(da.view, db.view, empty([130, 140], np.float32)))
    want = oracle.matmul(da.host_view(), db.host_view())
    assert np.isinf(want).any() and np.isnan(want).any()
    assert_bit_exact(got, want, "tf32x3 with non-finite inputs")
    # the same integers, all finite: the tensor-core path, exact for these values
    a[3, 5] = a[7, 1] = 1.0
    b[2, 9] = -2.0
    check(contiguous(a), contiguous(b))


def test_tf32x3_wide_tiles():
    """Shapes with at least six waves of 128 x 256 tiles take the wide tile:
    [4096, 40] x [40, 7000] has 32 x 28 such tiles, the last column of tiles
    88 wide; then the same shape through the exact path (a NaN input)."""
    import oracle
    from _util import assert_bit_exact
    from tensorrs_b200 import device
    a = rand([4096, 40], 51)
    b = rand([40, 7000], 52)
    worst = check(contiguous(a), contiguous(b))
    print(f"wide tiles: worst |gpu - ref| / sum|ab| = {worst:.2e}")
    a[100, 3] = np.nan
    da, db = contiguous(a), contiguous(b)
    got = to_host(device.matmul_tf32x3(da.view, db.view, empty([4096, 7000], np.float32)))
    assert_bit_exact(got, oracle.matmul(da.host_view(), db.host_view()), "wide tiles, exact path")


def test_tf32x3_at_the_benchmark_size():
    """[4096, 4096] x [4096, 4096] ~N(0,1), the measured configuration.  The
    reference's chain at this size comes from trs_matmul, which is bit-identical
    to it (test_matmul_gpu.py): every output within 1e-5 * sum_k |a_ik b_kj| of
    it, and within the worst case of an f32 accumulation of K split products,
    ((K - 1) 2^-24 + 2^-21) * sum_k |a_ik b_kj|, of the exact product (f64)."""
    import torch
    from tensorrs_b200 import device
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(61)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    va, vb = device.view_of(a), device.view_of(b)
    out = torch.empty(n, n, device="cuda")
    device.matmul_tf32x3(va, vb, out)
    ref = torch.empty(n, n, device="cuda")
    device.matmul(va, vb, ref)
    exact = a.double() @ b.double()
    mag = a.double().abs() @ b.double().abs()
    got = out.double()
    worst_ref = float(((got - ref.double()).abs() / mag).max())
    worst_exact = float(((got - exact).abs() / mag).max())
    assert worst_ref <= 1e-5, worst_ref
    assert worst_exact <= (n - 1) * 2.0**-24 + 2.0**-21, worst_exact
    print(f"4096^3: worst / sum|ab|: {worst_ref:.2e} against the reference's chain, {worst_exact:.2e} against exact")
