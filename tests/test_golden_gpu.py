"""Every known answer of the reference's own tests, computed on the GPU through
the C ABI."""
from __future__ import annotations

import numpy as np
import pytest

from _golden import check, storage_of
from conftest import NP_DTYPES, golden_cases

pytestmark = pytest.mark.gpu


def _run_gpu(case):
    from _gpu import DevView, empty, to_host
    from tensorrs_b200 import abi, device
    dt = NP_DTYPES[case["dtype"]]
    dvs = [DevView(storage_of(i, dt), i["shape"], i.get("strides"), i.get("offset", 0)) for i in case["inputs"]]
    op = case["op"]
    if op == "binary":
        shape = list(np.broadcast_shapes(tuple(dvs[0].shape), tuple(dvs[1].shape)))
        out = empty(shape, dt)
        before = [d.t.clone() for d in dvs]
        device.binary(case["binop"], dvs[0].view, dvs[1].view, out)
        if case["expect"].get("inputs_unchanged"):
            for d, b in zip(dvs, before):
                assert bool((d.t == b).all())
        return to_host(out)
    if op == "pack":
        out = empty(dvs[0].shape, dt)
        return to_host(device.pack(dvs[0].view, out))
    if op == "unary":
        out = empty(dvs[0].shape, dt)
        p = case.get("params", [0, 0])
        return to_host(device.unary(case["unop"], dvs[0].view, out, p[0], p[1]))
    if op == "sum":
        out = empty([1], dt)
        return to_host(device.sum_all(dvs[0].view, out))
    if op == "sum_axis":
        shape = list(dvs[0].shape)
        if case["keepdim"]:
            shape[case["axis"]] = 1
        else:
            shape.pop(case["axis"])
        out = empty(shape, dt)
        return to_host(device.sum_axis(dvs[0].view, case["axis"], case["keepdim"], out))
    if op in ("max_axis", "argmax_axis"):
        shape = list(dvs[0].shape)
        shape.pop(case["axis"])
        if op == "max_axis":
            return to_host(device.max_axis(dvs[0].view, case["axis"], empty(shape, dt)))
        return to_host(device.argmax_axis(dvs[0].view, case["axis"], empty(shape, np.int64)))
    if op == "reduce_broadcast_grad":
        out = empty(case["target"], dt)
        st = device.reduce_broadcast_grad(dvs[0].view, case["target"], out)
        return None if st == abi.NONE else to_host(out)
    if op == "softmax":
        out = empty(dvs[0].shape, dt)
        return to_host(device.softmax_lastdim(dvs[0].view, out))
    if op in ("max_pool2d", "avg_pool2d", "max_pool2d_backward"):
        kh, kw = case["kernel"]
        sh, sw = case["stride"]
        n, c, h, w = dvs[0].shape
        if op == "max_pool2d_backward":
            gx = empty([n, c, h, w], dt)
            return to_host(device.max_pool2d_backward(dvs[0].view, dvs[1].view, (kh, kw), gx, (sh, sw)))
        oh, ow = device.pooled_size((h, w), (kh, kw), (sh, sw))
        fn = device.max_pool2d if op == "max_pool2d" else device.avg_pool2d
        return to_host(fn(dvs[0].view, (kh, kw), empty([n, c, oh, ow], dt), (sh, sw)))
    if op == "layer_norm":
        return _layer_norm_gpu(dvs, case["epsilon"], dt)
    if op == "matmul":
        out = empty(device.matmul_shape(dvs[0].view, dvs[1].view), dt)
        return to_host(device.matmul(dvs[0].view, dvs[1].view, out))
    if op in ("unfold_2d", "unfold_fold_2d"):
        (kh, kw), (sh, sw), (ph, pw) = case["kernel"], case["stride"], case["padding"]
        n, c, h, w = dvs[0].shape
        oh, ow = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
        cols = device.unfold_2d(dvs[0].view, (kh, kw), (sh, sw), (ph, pw), empty([n * oh * ow, c * kh * kw], dt))
        if op == "unfold_2d":
            return to_host(cols)
        back = device.fold_2d(device.view_of(cols), (kh, kw), (sh, sw), (ph, pw), empty([n, c, h, w], dt))
        return to_host(back)
    raise ValueError(op)


def _layer_norm_gpu(dvs, eps, dt):
    """LayerNorm::forward (nn/layer_norm.rs:20-33) as the chain of calls it makes."""
    from _gpu import empty
    from tensorrs_b200 import device
    x, gamma, beta = dvs
    shape = x.shape
    n = shape[-1]
    axis = len(shape) - 1
    kd = list(shape[:-1]) + [1]
    s = device.sum_axis(x.view, axis, True, empty(kd, dt))
    mean = device.unary("div_scalar", device.view_of(s), empty(kd, dt), float(n))
    xm = device.binary("sub", x.view, device.view_of(mean), empty(shape, dt))
    sq = device.unary("pow_scalar", device.view_of(xm), empty(shape, dt), 2.0)
    v = device.sum_axis(device.view_of(sq), axis, True, empty(kd, dt))
    var = device.unary("div_scalar", device.view_of(v), empty(kd, dt), float(n))
    ve = device.unary("add_scalar", device.view_of(var), empty(kd, dt), eps)
    den = device.unary("pow_scalar", device.view_of(ve), empty(kd, dt), 0.5)
    xh = device.binary("div", device.view_of(xm), device.view_of(den), empty(shape, dt))
    xg = device.binary("mul", device.view_of(xh), gamma.view, empty(shape, dt))
    out = device.binary("add", device.view_of(xg), beta.view, empty(shape, dt))
    from _gpu import to_host
    return to_host(out)


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["name"])
def test_gpu_matches_reference_kat(case):
    check(case, _run_gpu(case))


@pytest.mark.parametrize("case", [c for c in golden_cases() if not c["expect"].get("none")],
                         ids=lambda c: c["name"])
def test_gpu_matches_oracle_on_kat_inputs(case):
    """Beyond the reference's assertion, the GPU result equals the oracle's."""
    from _golden import run_oracle
    from _util import assert_bit_exact, max_ulp
    got = np.asarray(_run_gpu(case))
    want = np.asarray(run_oracle(case))
    if case["op"] in ("binary", "pack", "max_axis", "argmax_axis", "max_pool2d", "avg_pool2d",
                      "max_pool2d_backward") or case["dtype"] in ("i32", "i64") \
            or (case["op"] == "unary" and case["unop"] in ("relu", "leaky_relu", "abs", "clamp", "mul_scalar")):
        assert_bit_exact(got, want, case["name"])
    elif case["op"] in ("sum", "sum_axis", "reduce_broadcast_grad"):
        assert np.allclose(got, want, rtol=1e-6, atol=0)
    elif case["op"] == "layer_norm":
        # a chain of ten calls with two sums and two powf: a few ulp
        assert max_ulp(got, want) <= 8, case["name"]
    else:
        assert max_ulp(got, want) <= 2, case["name"]
