"""Runs the reference's known-answer cases (tests/golden/reference_kats.json)
through the oracle or through the C ABI, and checks the expectations the
reference's own assertions make."""
from __future__ import annotations

import numpy as np

from conftest import NP_DTYPES


def storage_of(inp, dt) -> np.ndarray:
    """An input's storage: its listed values, or 1, 2, ..., n for a ramp
    (nn/pool.rs:245-248)."""
    if inp.get("ramp"):
        return np.arange(1, int(np.prod(inp["shape"])) + 1).astype(dt)
    return np.array(inp["storage"], dtype=dt)


def _host_views(case):
    import oracle
    dt = NP_DTYPES[case["dtype"]]
    vs = []
    for inp in case["inputs"]:
        st = storage_of(inp, dt)
        vs.append(oracle.HostView(st, inp["shape"], inp.get("strides"), inp.get("offset", 0)))
    return vs


def _layer_norm(run_bin, run_sum_axis, run_scalar, x, gamma, beta, eps):
    """LayerNorm::forward (nn/layer_norm.rs:20-33) as the chain of calls it makes."""
    axis = len(x.shape) - 1
    n = x.shape[axis]
    mean = run_scalar("div_scalar", run_sum_axis(x, axis, True), float(n))
    xm = run_bin("sub", x, mean)
    sq = run_scalar("pow_scalar", xm, 2.0)
    var = run_scalar("div_scalar", run_sum_axis(sq, axis, True), float(n))
    denom = run_scalar("pow_scalar", run_scalar("add_scalar", var, eps), 0.5)
    xhat = run_bin("div", xm, denom)
    return run_bin("add", run_bin("mul", xhat, gamma), beta)


def run_oracle(case):
    """Returns the result array, or None for a reference `None`."""
    import oracle
    vs = _host_views(case)
    op = case["op"]
    if op == "binary":
        return oracle.binary(case["binop"], vs[0], vs[1])
    if op == "pack":
        return oracle.unary("none", vs[0])
    if op == "unary":
        p = case.get("params", [0, 0])
        return oracle.unary(case["unop"], vs[0], p[0], p[1])
    if op == "sum":
        return np.array([oracle.sum_all(vs[0])])
    if op == "sum_axis":
        return oracle.sum_axis(vs[0], case["axis"], case["keepdim"])
    if op == "max_axis":
        return oracle.max_argmax_axis(vs[0], case["axis"])[0]
    if op == "argmax_axis":
        return oracle.max_argmax_axis(vs[0], case["axis"])[1]
    if op == "reduce_broadcast_grad":
        return oracle.reduce_broadcast_grad(vs[0], case["target"])
    if op == "softmax":
        return oracle.softmax_lastdim(vs[0])
    if op in ("max_pool2d", "avg_pool2d"):
        return oracle.pool2d(op[:3], vs[0], case["kernel"], case["stride"])
    if op == "max_pool2d_backward":
        return oracle.max_pool2d_backward(vs[0], vs[1], case["kernel"], case["stride"])
    if op == "matmul":
        return oracle.matmul(vs[0], vs[1])
    if op == "unfold_2d":
        return oracle.unfold_2d(vs[0], case["kernel"], case["stride"], case["padding"])
    if op == "unfold_fold_2d":  # the fold doctest folds the unfold of its input back
        cols = oracle.unfold_2d(vs[0], case["kernel"], case["stride"], case["padding"])
        return oracle.fold_2d(oracle.contiguous(cols), vs[0].shape, case["kernel"], case["stride"], case["padding"])
    if op == "layer_norm":
        wrap = oracle.contiguous
        return _layer_norm(
            lambda o, a, b: oracle.binary(o, wrap(a) if isinstance(a, np.ndarray) else a,
                                          wrap(b) if isinstance(b, np.ndarray) else b),
            lambda a, ax, kd: oracle.sum_axis(wrap(a) if isinstance(a, np.ndarray) else a, ax, kd),
            lambda o, a, s: oracle.unary(o, wrap(a) if isinstance(a, np.ndarray) else a, s),
            vs[0], vs[1], vs[2], case["epsilon"])
    raise ValueError(op)


def check(case, got):
    exp = case["expect"]
    name = case["name"]
    if exp.get("none"):
        assert got is None, f"{name}: expected None"
        return
    assert got is not None, f"{name}: got None"
    got = np.asarray(got)
    assert list(got.shape) == list(exp["shape"]), f"{name}: shape {got.shape} != {exp['shape']}"
    flat = got.reshape(-1)
    if "data" in exp:
        for i, w in enumerate(exp["data"]):
            if w is None:
                continue
            if exp.get("exact"):
                assert flat[i] == w, f"{name}[{i}]: {flat[i]!r} != {w!r}"
            else:
                assert abs(float(flat[i]) - w) < exp["approx"], f"{name}[{i}]: {flat[i]!r} vs {w!r}"
    for c in exp.get("checks", []):
        v = float(flat[c["index"]])
        if "lt" in c:
            assert v < c["lt"], f"{name}[{c['index']}] = {v}"
        if "ge" in c:
            assert v >= c["ge"], f"{name}[{c['index']}] = {v}"
    if exp.get("finite"):
        assert np.isfinite(flat).all(), name
    if "row_sum" in exp:
        assert abs(float(flat.astype(np.float64).sum()) - exp["row_sum"]) < exp["approx"], name
    if exp.get("increasing"):
        assert all(flat[i] < flat[i + 1] for i in range(len(flat) - 1)), name
