"""trs_elementwise_row_sums: the chain `y = prog(in); y.sum_axis(last);
y.sum()` (binary_op, ops.rs:240-300; sum_axis, base.rs:1051-1107; sum,
base.rs:1024-1030) in one pass, through the C ABI against the oracle.

y is compared bit for bit (within 2 ulp for sigmoid, whose f32 map is held to
that everywhere); the row sums and the total, accumulated in f64 and rounded
once, within 1e-5 * sum|y| of the reference's sequential fold and within
2^-23 |exact| + 2^-40 sum|y| of the exact sum (f64: n * 2^-52 sum|y| and
2^-51 |exact| + n * 2^-52 sum|y|); integers wrap and are compared exactly.
The fused kernel serves contiguous results of at least 256 rows whose inputs
run along the last axis or are constant along it; the other layouts take the
three separate passes, which are checked the same way.  The number of kernel
launches tells the two apart: two for the fused pass (the row kernel and the
total's fold), more for the three passes."""
from __future__ import annotations

import math

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact, max_ulp

pytestmark = pytest.mark.gpu


def rand(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.standard_normal(size=shape).astype(dtype)
    return rng.integers(-(2**30), 2**30, size=shape).astype(dtype)


def launches():
    from tensorrs_b200 import abi
    return int(abi.load().trs_launch_count())


def check_sums(got, ref, y: np.ndarray, axis_rows: bool):
    """got/ref: GPU and oracle sums of y over its last axis (axis_rows) or all of it."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if y.dtype.kind != "f":
        assert_bit_exact(got, ref, "integer sums wrap exactly")
        return
    yd = y.astype(np.float64)
    if axis_rows:
        sabs = np.abs(yd).sum(axis=-1).reshape(got.shape)
        exact = np.array([math.fsum(r) for r in yd.reshape(-1, y.shape[-1])]).reshape(got.shape)
        n = y.shape[-1]
    else:
        sabs = np.abs(yd).sum()
        exact = math.fsum(yd.ravel())
        n = y.size
    g = got.astype(np.float64)
    r = ref.astype(np.float64)
    if y.dtype == np.float32:
        tol_ref = 1e-5 * sabs
        tol_exact = np.abs(exact) * 2.0**-23 + 2.0**-40 * sabs
    else:
        tol_ref = n * 2.0**-52 * sabs
        tol_exact = np.abs(exact) * 2.0**-51 + n * 2.0**-52 * sabs
    assert np.all(np.abs(g - r) <= tol_ref + 1e-300), float(np.max(np.abs(g - r) - tol_ref))
    assert np.all(np.abs(g - exact) <= tol_exact + 1e-300)


def run_case(n_in, op1, op2, epi, views, keepdim=False, want_rows=True, want_total=True, fused=None):
    import oracle
    from tensorrs_b200 import abi, device
    hv = [v.host_view() for v in views]
    want_y = oracle.program(n_in, op1, op2, epi, hv)
    dtype = want_y.dtype
    y = empty(want_y.shape, dtype)
    rshape = list(want_y.shape[:-1]) + ([1] if keepdim else [])
    rows = empty(rshape, dtype) if want_rows else None
    total = empty([1], dtype) if want_total else None
    before = launches()
    device.elementwise_row_sums(abi.program(n_in, abi.BINOPS[op1], abi.BINOPS[op2], epi), [v.view for v in views],
                                y, rows, total)
    n_launch = launches() - before
    got_y = to_host(y)
    if epi == "sigmoid":
        assert max_ulp(got_y, want_y) <= 2
    else:
        assert_bit_exact(got_y, want_y, "y")
    # the sums are of the y the GPU produced (identical to the oracle's but for sigmoid)
    yv = oracle.contiguous(got_y)
    if want_rows:
        ref_rows = oracle.sum_axis(yv, got_y.ndim - 1, keepdim)
        check_sums(to_host(rows), ref_rows, got_y, True)
    if want_total:
        check_sums(to_host(total), np.array([oracle.sum_all(yv)]), got_y, False)
    if fused is not None:
        assert (n_launch == (2 if want_total else 1)) == fused, n_launch
    return n_launch


def test_config1_chain_in_one_pass():
    """Config 1 at its size, seed and distribution: A [1024, 1024] + b [1024]."""
    import oracle
    n = 1024
    a = oracle.fill_uniform(np.float32, n * n, 0).reshape(n, n)
    b = oracle.fill_uniform(np.float32, n, 0, first=n * n)
    run_case(2, "add", "add", "none", [contiguous(a), contiguous(b)], fused=True)


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64], ids=lambda d: np.dtype(d).name)
def test_row_bias_add_every_dtype(dtype):
    run_case(2, "add", "add", "none", [contiguous(rand([512, 1000], dtype, 1)), contiguous(rand([1000], dtype, 2))],
             fused=True)


def test_column_broadcast_and_odd_rows():
    """b [300, 1] is constant along each row (one value per row); rows of 77
    elements take the element-by-element form."""
    run_case(2, "sub", "add", "none", [contiguous(rand([300, 77], np.float32, 3)),
                                       contiguous(rand([300, 1], np.float32, 4))], fused=True)


def test_three_inputs_and_leading_dims():
    """X [6, 64, 48] & s [48] + c [6, 64, 1]: the leading dimensions step as one
    row index for every input (c: one value per row)."""
    run_case(3, "mul", "add", "none", [contiguous(rand([6, 64, 48], np.float64, 5)),
                                       contiguous(rand([48], np.float64, 6)),
                                       contiguous(rand([6, 64, 1], np.float64, 7))], fused=True)


def test_integer_wrap_keepdim_rows_only():
    run_case(2, "mul", "add", "none", [contiguous(rand([256, 64], np.int32, 8)),
                                       contiguous(rand([256, 64], np.int32, 9))],
             keepdim=True, want_total=False, fused=True)
    run_case(2, "sub", "add", "none", [contiguous(rand([1024, 16], np.int64, 10)),
                                       contiguous(rand([1024, 16], np.int64, 11))], fused=True)


def test_sigmoid_program_total_only():
    run_case(1, "add", "add", "sigmoid", [contiguous(rand([400, 256], np.float32, 12))], want_rows=False,
             fused=True)


def test_layouts_that_take_the_three_passes():
    # fewer than 256 rows
    run_case(2, "add", "add", "none", [contiguous(rand([100, 64], np.float32, 13)),
                                       contiguous(rand([64], np.float32, 14))], fused=False)
    # a transposed input (runs along the rows, not the last axis)
    at = rand([256, 512], np.float32, 15)
    run_case(2, "add", "add", "none", [DevView(at, [512, 256], [1, 512], 0),
                                       contiguous(rand([256], np.float32, 16))], fused=False)
    # s [6, 1, 48] is constant along the middle dimension: no single row stride
    run_case(3, "mul", "add", "none", [contiguous(rand([6, 64, 48], np.float32, 17)),
                                       contiguous(rand([6, 1, 48], np.float32, 18)),
                                       contiguous(rand([48], np.float32, 19))], fused=False)
    # integer division reports a zero divisor through the separate pass
    run_case(2, "div", "add", "none", [contiguous(rand([512, 8], np.int32, 20)),
                                       contiguous(np.full([8], 7, np.int32))], fused=False)


def test_empty_rows_and_errors():
    from tensorrs_b200 import abi, device
    x = contiguous(np.zeros([0, 5], np.float32))
    rows = empty([0], np.float32)
    total = empty([1], np.float32)
    device.elementwise_row_sums(abi.program(1), [x.view], empty([0, 5], np.float32), rows, total)
    assert to_host(total)[0] == 0.0 and not np.signbit(to_host(total)[0])
    a = contiguous(rand([300, 8], np.float32, 21))
    y = empty([300, 8], np.float32)
    with pytest.raises(abi.TrsError) as e:
        device.elementwise_row_sums(abi.program(1), [a.view], y, None, None)
    assert e.value.status == abi.ERR_ARG
    with pytest.raises(abi.TrsError) as e:  # row sums of the wrong shape
        device.elementwise_row_sums(abi.program(1), [a.view], y, empty([8], np.float32), None)
    assert e.value.status == abi.ERR_SHAPE
    with pytest.raises(abi.TrsError) as e:  # the total inside y
        device.elementwise_row_sums(abi.program(1), [a.view], y, None, y[0, :1])
    assert e.value.status == abi.ERR_ALIAS
    with pytest.raises(abi.TrsError) as e:
        device.elementwise_row_sums(abi.program(2, abi.ADD), [a.view, contiguous(rand([7], np.float32, 22)).view],
                                    y, None, total)
    assert "!!!Add: incompatible shapes!!!" in e.value.message
