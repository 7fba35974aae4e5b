"""K-EW parity: broadcast element-wise ops over strided views, on the GPU
through the C ABI, against the oracle on the same seeded inputs.

Tolerances (written here, from the contract): add/sub/mul/div, ReLU/LeakyReLU,
abs/neg/sign/clamp and the scalar operators are bit-exact (any NaN matches any
NaN); transcendental results (sigmoid, tanh, ELU, SELU, E^x, ln, powf) are
within 2 ulp of the oracle's glibc values."""
from __future__ import annotations

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact, max_ulp, ulp_diff

pytestmark = pytest.mark.gpu

DTYPES = [np.float32, np.float64, np.int32, np.int64]


def rand(shape, dtype, seed, lo=-4.0, hi=4.0):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.uniform(lo, hi, size=shape).astype(dtype)
    return rng.integers(-1000, 1000, size=shape).astype(dtype)


def special_f32(n, seed):
    """N(0,1) values salted with the special values the reference's rules touch."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32) * 4
    sp = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-38, -1e-38, 88.0, 89.0, -88.0,
                   -104.0, 100.0, -100.0, 400.0, -400.0, 20.0, -20.0, 1.0, -1.0, 3e38, -3e38], dtype=np.float32)
    x[: sp.size] = sp
    return x


def gpu_binary(op, a: DevView, b: DevView, dtype):
    from tensorrs_b200 import device
    shape = list(np.broadcast_shapes(tuple(a.shape), tuple(b.shape)))
    out = empty(shape, dtype)
    device.binary(op, a.view, b.view, out)
    return to_host(out)


BCAST_SHAPES = [
    ([37], [37]), ([1], [53]), ([3, 4, 5], [4, 1]), ([64, 1], [1, 48]), ([2, 3, 1, 5], [7, 1]),
    ([1024, 1024], [1024]), ([5, 1, 6, 1, 7, 2], [1, 3, 1, 4, 1, 2]), ([0, 4], [0, 4]), ([256, 130], [130]),
]


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("sa,sb", BCAST_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_binary_broadcast_bit_exact(op, sa, sb, dtype):
    a = rand(sa, dtype, 1)
    b = rand(sb, dtype, 2)
    if op == "div" and np.dtype(dtype).kind == "i":
        b[b == 0] = 7
    da, db = contiguous(a), contiguous(b)
    import oracle
    want = oracle.binary(op, da.host_view(), db.host_view())
    got = gpu_binary(op, da, db, dtype)
    assert_bit_exact(got, want, f"{op} {sa} {sb}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_powf_within_two_ulp(dtype):
    rng = np.random.default_rng(5)
    a = np.abs(rng.standard_normal(4096)).astype(dtype) * 3
    b = rng.uniform(-6, 6, 4096).astype(dtype)
    a[:8] = [0.0, -2.0, -2.0, 1.0, 2.718281828, 10.0, 0.5, -0.0]
    b[:8] = [0.0, 3.0, 0.5, np.nan, -3.0, 50.0, -200.0, -1.0]
    da, db = contiguous(a), contiguous(b)
    import oracle
    want = oracle.binary("pow", da.host_view(), db.host_view())
    got = gpu_binary("pow", da, db, dtype)
    assert max_ulp(got, want) <= 2


def test_transposed_operand_tile_kernel_bit_exact():
    """config 2 in small: A & B^T with B^T a strided view, odd sizes."""
    import oracle
    for n, m in [(4096, 4096), (97, 131), (33, 32), (1, 40)]:
        a = rand([n, m], np.float32, 3)
        b = rand([m, n], np.float32, 4)
        da = contiguous(a)
        dbt = DevView(b.reshape(-1), [n, m], [1, n], 0)
        want = oracle.binary("mul", da.host_view(), dbt.host_view())
        got = gpu_binary("mul", da, dbt, np.float32)
        assert_bit_exact(got, want, f"A & B^T {n}x{m}")


def test_transposed_batched_operands():
    import oracle
    # [B, n, m] + permuted view of a [B, m, n] storage, plus a broadcast row
    a = rand([3, 40, 72], np.float64, 5)
    b = rand([3, 72, 40], np.float64, 6)
    da = contiguous(a)
    dbt = DevView(b.reshape(-1), [3, 40, 72], [72 * 40, 1, 40], 0)
    want = oracle.binary("sub", da.host_view(), dbt.host_view())
    assert_bit_exact(gpu_binary("sub", da, dbt, np.float64), want)


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("n,m", [(4096, 4096), (300, 4100), (64, 64), (8, 1000), (1000, 8), (132, 68)],
                         ids=lambda v: str(v))
def test_transposed_vectorised_tiles(n, m, dtype):
    """A op B^T on the vectorised tile path (row starts 16-byte aligned):
    full and partial tiles, several ops, bit-exact."""
    import oracle
    a = rand([n, m], dtype, 31)
    b = rand([m, n], dtype, 32)
    da = contiguous(a)
    dbt = DevView(b.reshape(-1), [n, m], [1, n], 0)
    for op in ("mul", "add", "sub"):
        want = oracle.binary(op, da.host_view(), dbt.host_view())
        assert_bit_exact(gpu_binary(op, da, dbt, dtype), want, f"{op} {n}x{m}")
    # B^T op A: the transposed input first
    want = oracle.binary("mul", dbt.host_view(), da.host_view())
    assert_bit_exact(gpu_binary("mul", dbt, da, dtype), want, "B^T & A")


def test_transposed_pack_sigmoid_and_three_inputs():
    """get_data of a transposed view (trs_pack), sigmoid(A & B^T) fused (the
    config-2 program), and a 3-input program mixing two transposed inputs with
    a per-row column vector plus the sum epilogue, on the vectorised tile path."""
    import oracle
    from tensorrs_b200 import abi, device
    n = 1024
    a = rand([n, n], np.float32, 41)
    b = rand([n, n], np.float32, 42)
    c = rand([n, 1], np.float32, 43)
    da, dc = contiguous(a), contiguous(c)
    dbt = DevView(b.reshape(-1), [n, n], [1, n], 0)
    dat = DevView(a.reshape(-1), [n, n], [1, n], 0)
    got = to_host(device.pack(dbt.view, empty([n, n], np.float32)))
    assert_bit_exact(got, np.ascontiguousarray(b.T), "pack of B^T")
    prog = abi.program(2, abi.MUL, epilogue="sigmoid")
    out = empty([n, n], np.float32)
    device.elementwise(prog, [da.view, dbt.view], out)
    want = oracle.program(2, "mul", "add", "sigmoid", [da.host_view(), dbt.host_view()])
    assert max_ulp(to_host(out), want) <= 2
    prog3 = abi.program(3, abi.MUL, abi.ADD)
    out3 = empty([n, n], np.float32)
    s3 = empty([1], np.float32)
    device.elementwise(prog3, [dat.view, dbt.view, dc.view], out3, s3)
    want3 = oracle.program(3, "mul", "add", "none", [dat.host_view(), dbt.host_view(), dc.host_view()])
    assert_bit_exact(to_host(out3), want3, "A^T & B^T + c")
    ref_s = oracle.sum_all(oracle.contiguous(want3))
    exact, sabs = oracle.sum_f64(oracle.contiguous(want3))
    got_s = float(to_host(s3)[0])
    assert abs(got_s - ref_s) <= 1e-5 * sabs and abs(got_s - exact) <= abs(exact) * 2.0**-23 + 2.0**-40 * sabs


@pytest.mark.parametrize("n,m", [(512, 512), (136, 200)], ids=lambda v: str(v))
def test_both_operands_transposed(n, m):
    """A^T & B^T and sigmoid(A^T & B^T): both inputs read through shared-memory
    tiles (full and partial tiles), bit-exact for the product and within
    2 ulp for the sigmoid."""
    import oracle
    from tensorrs_b200 import abi, device
    a = rand([m, n], np.float32, 61)
    b = rand([m, n], np.float32, 62)
    dat = DevView(a.reshape(-1), [n, m], [1, n], 0)
    dbt = DevView(b.reshape(-1), [n, m], [1, n], 0)
    want = oracle.binary("mul", dat.host_view(), dbt.host_view())
    assert_bit_exact(gpu_binary("mul", dat, dbt, np.float32), want, "A^T & B^T")
    out = empty([n, m], np.float32)
    device.elementwise(abi.program(2, abi.MUL, epilogue="sigmoid"), [dat.view, dbt.view], out)
    want = oracle.program(2, "mul", "add", "sigmoid", [dat.host_view(), dbt.host_view()])
    assert max_ulp(to_host(out), want) <= 2


def test_transposed_batched_vectorised():
    """[B, n, m] with a permuted view of a [B, m, n] storage, 16-byte aligned."""
    import oracle
    a = rand([3, 128, 72], np.float32, 51)
    b = rand([3, 72, 128], np.float32, 52)
    da = contiguous(a)
    dbt = DevView(b.reshape(-1), [3, 128, 72], [72 * 128, 1, 128], 0)
    want = oracle.binary("mul", da.host_view(), dbt.host_view())
    assert_bit_exact(gpu_binary("mul", da, dbt, np.float32), want)


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
def test_reversed_offset_and_gapped_views(dtype):
    """step_slice views: negative steps, offsets and gaps (base.rs:369-398)."""
    import oracle
    st = rand([600], dtype, 7)
    cases = [
        ([100], [-1], 599),            # reversed
        ([10, 10], [30, 3], 2),        # gapped
        ([12, 5], [-40, 7], 480),      # reversed rows, gapped columns
        ([6, 4, 3], [1, -6, 50], 18),  # mixed signs
    ]
    for shape, strides, off in cases:
        dv = DevView(st, shape, strides, off)
        other = rand(shape, dtype, 8)
        do = contiguous(other)
        want = oracle.binary("add", dv.host_view(), do.host_view())
        assert_bit_exact(gpu_binary("add", dv, do, dtype), want, f"{shape} {strides} {off}")
        want = oracle.unary("none", dv.host_view())
        from tensorrs_b200 import device
        got = to_host(device.pack(dv.view, empty(shape, dtype)))
        assert_bit_exact(got, want, "pack")


def test_zero_stride_scalar_operand():
    """Tensor::scalar has shape [1], stride [0] (base.rs:212-219)."""
    import oracle
    a = rand([9, 11], np.float32, 9)
    s = DevView(np.array([2.5], np.float32), [1], [0], 0)
    da = contiguous(a)
    for op in ["add", "sub", "mul", "div"]:
        want = oracle.binary(op, da.host_view(), s.host_view())
        assert_bit_exact(gpu_binary(op, da, s, np.float32), want, op)
        want = oracle.binary(op, s.host_view(), da.host_view())
        assert_bit_exact(gpu_binary(op, s, da, np.float32), want, op + " reversed")


EXACT_UNARY = [("neg", 0, 0), ("relu", 0, 0), ("leaky_relu", 0.1, 0), ("abs", 0, 0), ("sign", 0, 0),
               ("clamp", -1.5, 2.25), ("add_scalar", 0.3, 0), ("sub_scalar", 0.3, 0), ("rsub_scalar", 0.3, 0),
               ("mul_scalar", 1.7, 0), ("div_scalar", 3.0, 0)]
ULP_UNARY = [("sigmoid", 0, 0), ("tanh", 0, 0), ("exp", 0, 0), ("ln", 0, 0), ("pow_scalar", 2.0, 0),
             ("pow_scalar", 0.5, 0), ("rpow_scalar", 2.7182817, 0)]
# ELU / SELU compute (E^x - 1) * alpha * mask (elu.rs:58-62), which cancels
# near x = 0: an E^x within 2 ulp moves the result by up to 2 ulp of E^x
# times alpha (times lambda for SELU), far more than 2 ulp of the result.
CANCEL_UNARY = [("elu", 1.0, 0), ("elu", 0.5, 0), ("selu", 1.67326, 1.0507)]
# f64 transcendentals use CUDA's f64 library against glibc's f64 library.
F64_ULP = 4
@pytest.mark.parametrize("op,p0,p1", EXACT_UNARY, ids=lambda v: str(v))
@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_exact_unary_maps(op, p0, p1, dtype):
    import oracle
    from tensorrs_b200 import device
    x = special_f32(70001, 11).astype(dtype)
    dx = contiguous(x)
    want = oracle.unary(op, dx.host_view(), p0, p1)
    got = to_host(device.unary(op, dx.view, empty(x.shape, dtype), p0, p1))
    assert_bit_exact(got, want, op)


@pytest.mark.parametrize("op,p0,p1", ULP_UNARY, ids=lambda v: str(v))
@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_transcendental_unary_maps_within_two_ulp(op, p0, p1, dtype):
    import oracle
    from tensorrs_b200 import device
    x = special_f32(200003, 12).astype(dtype)
    if op in ("ln",):
        x = np.abs(x)
    dx = contiguous(x)
    want = oracle.unary(op, dx.host_view(), p0, p1)
    got = to_host(device.unary(op, dx.view, empty(x.shape, dtype), p0, p1))
    u = max_ulp(got, want)
    exact = int((ulp_diff(got, want) == 0).sum())
    print(f"{op} {np.dtype(dtype).name}: max {u} ulp, {exact}/{x.size} bit-identical")
    assert u <= (2 if dtype == np.float32 else F64_ULP), f"{op}: {u} ulp"


@pytest.mark.parametrize("op", ["exp", "sigmoid"])
def test_f32_exponentials_dense_sweep(op):
    """powf(E, x) (elu.rs:58-60) and sigmoid (autodiff/ops.rs:586-593) on 2^22
    points spanning every f32 result from overflow down through the
    subnormals to 0, plus the specials.  The exponential is within 1 ulp of
    glibc's (bit-identical for about 99 % of inputs of this spread; the host
    test of exp_f32.h measures every f32); sigmoid divides two quantities
    that both carry it (e / (1 + e)), so a one-ulp e can move it by 2 ulp."""
    import oracle
    from tensorrs_b200 import device
    x = np.linspace(-110.0, 95.0, 1 << 22).astype(np.float32)
    x = np.concatenate([x, np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 88.72283, 88.72284, -103.27893,
                                     -103.97208, -87.33655, 1e-30, -1e-30], np.float32)])
    dx = contiguous(x)
    want = oracle.unary(op, dx.host_view())
    got = to_host(device.unary(op, dx.view, empty(x.shape, np.float32)))
    u = max_ulp(got, want)
    exact = int((ulp_diff(got, want) == 0).sum())
    print(f"{op}: max {u} ulp, {exact}/{x.size} bit-identical")
    assert u <= (1 if op == "exp" else 2), f"{op}: {u} ulp"
    assert exact >= 0.99 * x.size


@pytest.mark.parametrize("op,p0,p1", CANCEL_UNARY, ids=lambda v: str(v))
@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_elu_selu(op, p0, p1, dtype):
    """ELU / SELU compose (E^x - 1) * alpha (* lambda) under masks (elu.rs:43-64,
    selu.rs:48-71).  The transcendental in them, E^x, is within one ulp of the
    reference's: for f32 it is the f64 evaluation rounded once (correctly
    rounded), and glibc's powf is within 0.82 ulp, so the two differ by at
    most one ulp and agree for almost every input; for f64 it is CUDA's pow,
    within 2 ulp of glibc's pow.  Subtracting 1 turns that ulp of E^x into
    many ulps of a result near 0, the reference's own rounding included, so
    the composed result is held to the bound this implies: K ulp of E^x times
    alpha (times lambda), plus 2 ulp of the result (K = 1 for f32, F64_ULP for
    f64).  f32 is checked over the specials and a dense sweep of the band
    x in [-4, 0] where E^x - 1 cancels, and must be bit-identical for at
    least 99.9 % of them."""
    import oracle
    from tensorrs_b200 import device
    x = special_f32(200003, 13).astype(dtype)
    if dtype == np.float32:
        band = np.linspace(-4.0, 0.0, 1 << 22, dtype=np.float32)
        tiny = -np.logspace(-38, -1, 1 << 16).astype(np.float32)
        x = np.concatenate([x, band, tiny])
    dx = contiguous(x)
    want = oracle.unary(op, dx.host_view(), p0, p1)
    got = to_host(device.unary(op, dx.view, empty(x.shape, dtype), p0, p1))
    ex = oracle.unary("exp", dx.host_view())  # E^x as the reference computes it
    scale = abs(p0) * (p1 if op == "selu" else 1.0)
    k = 1 if dtype == np.float32 else F64_ULP
    with np.errstate(invalid="ignore", over="ignore"):
        bound = k * scale * np.spacing(np.abs(ex)).astype(np.float64) + 2 * np.spacing(np.abs(want)).astype(np.float64)
        diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    ok = (np.isnan(got) & np.isnan(want)) | (got == want) | (diff <= bound)
    assert ok.all(), f"{op}: {(~ok).sum()} outside the bound, e.g. x={x[~ok][:3]}"
    same = float((ulp_diff(got, want) == 0).mean())
    print(f"{op} {np.dtype(dtype).name}: {same:.5%} bit-identical, max {max_ulp(got, want)} ulp of the result")
    if dtype == np.float32:
        assert same >= 0.999
    # x > 0 takes the exact branch: the value itself (NaN once E^x overflows)
    pos = (x > 0) & np.isfinite(want)
    assert_bit_exact(got[pos], want[pos], op + " positive branch")


def test_relu_keeps_negative_zero_and_nan():
    from tensorrs_b200 import device
    x = np.array([-2.0, -0.0, 0.0, np.nan, np.inf, -np.inf, 3.0], np.float32)
    got = to_host(device.unary("relu", contiguous(x).view, empty(x.shape, np.float32)))
    assert np.signbit(got[0]) and got[0] == 0 and np.signbit(got[1])
    assert not np.signbit(got[2]) and np.isnan(got[3]) and got[4] == np.inf
    assert np.isnan(got[5])  # -inf * 0 in the mask multiply
    assert got[6] == 3.0


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
def test_scalar_ops_on_all_dtypes(dtype):
    import oracle
    from tensorrs_b200 import device
    x = rand([1000], dtype, 13)
    dx = contiguous(x)
    for op, p in [("add_scalar", 3), ("sub_scalar", 3), ("rsub_scalar", 3), ("mul_scalar", -3),
                  ("div_scalar", 3), ("neg", 0), ("abs", 0)]:
        want = oracle.unary(op, dx.host_view(), p)
        got = to_host(device.unary(op, dx.view, empty(x.shape, dtype), p))
        assert_bit_exact(got, want, op)


def test_integer_wraparound_matches_release_build():
    import oracle
    a = np.array([2**31 - 1, -2**31, 123456789], np.int32)
    b = np.array([1, -1, 1000], np.int32)
    da, db = contiguous(a), contiguous(b)
    for op in ["add", "sub", "mul"]:
        assert_bit_exact(gpu_binary(op, da, db, np.int32), oracle.binary(op, da.host_view(), db.host_view()), op)


def test_integer_division_by_zero_is_an_error():
    from tensorrs_b200 import abi
    a = contiguous(np.array([1, 2, 3], np.int32))
    b = contiguous(np.array([1, 0, 3], np.int32))
    with pytest.raises(abi.TrsError) as e:
        gpu_binary("div", a, b, np.int32)
    assert e.value.status == abi.ERR_DIV_ZERO
    a = contiguous(np.array([-2**31], np.int32))
    b = contiguous(np.array([-1], np.int32))
    with pytest.raises(abi.TrsError) as e:
        gpu_binary("div", a, b, np.int32)
    assert "overflow" in e.value.message


PROGRAMS = [
    # (n_in, op1, op2, epilogue, p0, p1, shapes)
    (3, "mul", "add", "none", 0, 0, [[256, 512], [256, 512], [512]]),          # config 5 in small
    (3, "mul", "add", "relu", 0, 0, [[4, 16, 7, 9], [1, 16, 1, 1], [1, 16, 1, 1]]),  # config 4 in small
    (2, "mul", "add", "sigmoid", 0, 0, [[64, 80], [64, 80]]),                  # config 2 epilogue
    (2, "sub", "add", "tanh", 0, 0, [[33, 17], [17]]),
    (2, "add", "add", "elu", 1.0, 0, [[40, 40], [1, 40]]),
    (3, "div", "sub", "leaky_relu", 0.01, 0, [[10, 20], [20], [10, 1]]),
]


@pytest.mark.parametrize("prog", PROGRAMS, ids=lambda p: f"{p[1]}-{p[2]}-{p[3]}")
def test_fused_programs_equal_the_unfused_chain(prog):
    import oracle
    from tensorrs_b200 import abi, device
    n_in, op1, op2, epi, p0, p1, shapes = prog
    arrs = [rand(s, np.float32, 20 + i, -2, 2) for i, s in enumerate(shapes)]
    if op1 == "div":
        arrs[1][np.abs(arrs[1]) < 0.1] = 0.5
    dvs = [contiguous(a) for a in arrs]
    want = oracle.program(n_in, op1, op2, epi, [d.host_view() for d in dvs], p0, p1)
    out = empty(want.shape, np.float32)
    device.elementwise(abi.program(n_in, abi.BINOPS[op1], abi.BINOPS[op2], epi, p0, p1), [d.view for d in dvs], out)
    got = to_host(out)
    if epi in ("none", "relu", "leaky_relu"):
        assert_bit_exact(got, want, str(prog))
    else:
        assert max_ulp(got, want) <= 2


def test_fused_sum_epilogue_matches_sequential_sum_within_bound():
    """Y = A & B + c and sum(Y): Y bit-exact, the sum within 1e-5 * sum|y| of the
    reference's sequential f32 fold, and within the f64-accumulation bound of the
    exact sum."""
    import oracle
    from tensorrs_b200 import abi, device
    rows, cols = 512, 4096
    a = oracle.fill_uniform(np.float32, rows * cols, 4).reshape(rows, cols)
    b = oracle.fill_uniform(np.float32, rows * cols, 5).reshape(rows, cols)
    c = oracle.fill_uniform(np.float32, cols, 6)
    dvs = [contiguous(a), contiguous(b), contiguous(c)]
    out = empty([rows, cols], np.float32)
    s = empty([1], np.float32)
    device.elementwise(abi.program(3, abi.MUL, abi.ADD), [d.view for d in dvs], out, s)
    y = to_host(out)
    want_y = oracle.program(3, "mul", "add", "none", [d.host_view() for d in dvs])
    assert_bit_exact(y, want_y)
    ref = np.float64(oracle.sum_all(oracle.contiguous(want_y)))
    exact, sabs = oracle.sum_f64(oracle.contiguous(want_y))
    got = np.float64(to_host(s)[0])
    assert abs(got - ref) <= 1e-5 * sabs
    n = y.size
    assert abs(got - exact) <= 0.5 * np.spacing(np.float32(abs(exact))) + n * 2.0**-53 * sabs


def test_device_uniform_generator_equals_host_generator():
    import oracle
    from tensorrs_b200 import device
    for n, seed in [(1000, 0), (1 << 20, 4)]:
        t = empty([n], np.float32)
        device.fill_uniform(t, seed)
        assert_bit_exact(to_host(t), oracle.fill_uniform(np.float32, n, seed))
    t = empty([4096], np.float32)
    device.fill_uniform(t, 3, 0.5, 1.5)
    assert_bit_exact(to_host(t), oracle.fill_uniform(np.float32, 4096, 3, 0.5, 1.5))


def test_empty_tensors():
    from tensorrs_b200 import abi, device
    a = contiguous(np.zeros([0, 4], np.float32))
    out = empty([0, 4], np.float32)
    device.binary("add", a.view, a.view, out)
    s = empty([1], np.float32)
    device.sum_all(a.view, s)
    assert to_host(s)[0] == 0.0


def test_zero_dim_broadcast_fails_like_the_reference():
    """broadcast_shape maps (0, 1) to 1 (ops.rs:33-39), so broadcast_to then
    fails and the reference panics; the library reports the same text."""
    import oracle
    from tensorrs_b200 import abi
    a = contiguous(np.zeros([0, 4], np.float32))
    b = contiguous(np.ones([4], np.float32))
    with pytest.raises(oracle.OracleError) as oe:
        oracle.binary("add", a.host_view(), b.host_view())
    with pytest.raises(abi.TrsError) as ge:
        gpu_binary("add", a, b, np.float32)
    assert oe.value.message == ge.value.message == "broadcast_to failed (bug)"


def test_packed_sigmoid_equals_the_scalar_form():
    """The contiguous 1-D map and the transposed-tile multiply take sigmoid two
    elements at a time on packed f32x2 operations; a strided layout takes the
    scalar form.  The two perform the same roundings, so they agree bit for bit."""
    import oracle
    from tensorrs_b200 import abi, device
    x = np.concatenate([special_f32(100003, 21), np.linspace(-110.0, 95.0, 1 << 20).astype(np.float32)])
    n = x.size
    flat = contiguous(x)
    packed = to_host(device.unary("sigmoid", flat.view, empty([n], np.float32)))
    spread = np.zeros(2 * n, np.float32)
    spread[::2] = x
    strided = DevView(spread, [n], [2], 0)
    scalar = to_host(device.unary("sigmoid", strided.view, empty([n], np.float32)))
    assert_bit_exact(packed, scalar, "packed vs scalar sigmoid")
    assert max_ulp(packed, oracle.unary("sigmoid", flat.host_view())) <= 2
    # sigmoid(A & B^T): the 2-D tile kernel (packed) against a gapped B^T view
    # (scalar, one element per thread)
    m = 512
    a = special_f32(m * m, 22).reshape(m, m)
    b = special_f32(m * m, 23).reshape(m, m)
    da = contiguous(a)
    db = contiguous(b)
    db.shape, db.strides = [m, m], [1, m]
    prog = abi.program(2, abi.MUL, epilogue="sigmoid")
    y1 = empty([m, m], np.float32)
    device.elementwise(prog, [da.view, db.view], y1)
    gap = np.zeros((m, m + 3), np.float32)
    gap[:, :m] = b
    dg = DevView(gap, [m, m], [1, m + 3], 0)
    y2 = empty([m, m], np.float32)
    device.elementwise(prog, [da.view, dg.view], y2)
    assert_bit_exact(to_host(y1), to_host(y2), "packed vs scalar sigmoid(A & B^T)")
