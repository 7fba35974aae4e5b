"""Callers of the path fused into one kernel each, on the GPU through the C
ABI, against the oracle:

* the optimiser steps SGD (optim/sgd.rs:29-37), RMSprop (optim/rmsprop.rs:30-46)
  and Adam (optim/adam.rs:119-144): bit-exact against the reference's chain
  of tensor calls (oracle.opt_step) over several consecutive steps, with
  zeros, signed zeros, tiny and huge gradients, odd sizes (a scalar tail) and
  f32/f64;
* LayerNorm::forward (nn/layer_norm.rs:20-33): its sums accumulate in f64
  and round once, so against a restatement with exactly rounded sums (the
  `ideal` below: the kernel's own order of f32 operations, sums by fsum) the
  result is bit-identical except where an f64 sum rounds to the other f32
  neighbour (a handful of rows at most, checked to 1e-5 relative); against
  the reference's chain (f32 sequential sums, powf) it differs by the
  reference's own summation error, bounded in the test; and it meets the
  reference's known answers.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from _gpu import DevView, contiguous, empty, to_host
from _util import assert_bit_exact, max_ulp

pytestmark = pytest.mark.gpu


def _grads(rng, n, dtype):
    g = (rng.standard_normal(n) * 0.1).astype(dtype)
    g[:6] = np.array([0.0, -0.0, 1e-30, -1e-30, 3.0, -2.5])[:min(6, n)]
    return g


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("kind", ["sgd", "rmsprop", "adam"])
@pytest.mark.parametrize("n", [1, 7, 4096, 1000003, 1 << 22])
def test_optimiser_steps_bit_exact(kind, n, dtype):
    import torch

    import oracle
    from tensorrs_b200 import device
    rng = np.random.default_rng(n + len(kind))
    p = rng.standard_normal(n).astype(dtype)
    m = np.zeros(n, dtype)
    v = np.zeros(n, dtype)
    dp, dm, dv = (torch.from_numpy(a.copy()).cuda() for a in (p, m, v))
    alpha = 0.99
    for t in range(1, 4):
        g = _grads(rng, n, dtype)
        dg = torch.from_numpy(g).cuda()
        if kind == "sgd":
            device.sgd_step(dp, dg, 0.05)
            oracle.opt_step("sgd", p, g, None, None, 0.05)
        elif kind == "rmsprop":
            device.rmsprop_step(dp, dg, dv, 0.01, alpha, 1e-8)
            oracle.opt_step("rmsprop", p, g, None, v, 0.01, 0.9, alpha, 1e-8)
        else:
            device.adam_step(dp, dg, dm, dv, 0.01, t)
            oracle.opt_step("adam", p, g, m, v, 0.01, 0.9, 0.999, 1e-8, t)
        assert_bit_exact(to_host(dp), p, f"{kind} param, step {t}")
        if kind == "adam":
            assert_bit_exact(to_host(dm), m, f"adam m, step {t}")
        if kind != "sgd":
            assert_bit_exact(to_host(dv), v, f"{kind} v, step {t}")


def test_optimiser_step_errors():
    import torch

    from tensorrs_b200 import abi, device
    p = torch.zeros(64, 64, device="cuda")
    with pytest.raises(abi.TrsError) as e:
        device.sgd_step(p.t(), torch.zeros(64, 64, device="cuda"), 0.1)
    assert e.value.status == abi.ERR_VIEW
    with pytest.raises(abi.TrsError) as e:
        device.sgd_step(p, torch.zeros(64, 63, device="cuda"), 0.1)
    assert e.value.status == abi.ERR_SHAPE
    with pytest.raises(abi.TrsError) as e:
        device.adam_step(p, torch.zeros_like(p), torch.zeros_like(p), torch.zeros_like(p), 0.1, 0)
    assert e.value.status == abi.ERR_ARG
    with pytest.raises(abi.TrsError) as e:
        device.sgd_step(p, torch.zeros(64, 64, device="cuda", dtype=torch.float64), 0.1)
    assert e.value.status == abi.ERR_DTYPE


def _ideal_layer_norm(x2: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float) -> np.ndarray:
    """The kernel's order of operations in the element type, with the two
    sums exactly rounded (fsum) instead of accumulated in f64."""
    T = x2.dtype.type
    F = x2.shape[1]
    out = np.empty_like(x2)
    for r in range(x2.shape[0]):
        row = x2[r]
        mean = T(T(math.fsum(row.astype(np.float64))) / T(F))
        xm = row - mean
        sq = xm * xm
        var = T(T(math.fsum(sq.astype(np.float64))) / T(F))
        denom = np.sqrt(T(var + T(eps)))
        out[r] = (xm / denom) * gamma + beta
    return out


def _chain_layer_norm(x, gamma, beta, eps):
    import oracle
    from _golden import _layer_norm
    wrap = oracle.contiguous
    return _layer_norm(
        lambda o, a, b: oracle.binary(o, wrap(a) if isinstance(a, np.ndarray) else a,
                                      wrap(b) if isinstance(b, np.ndarray) else b),
        lambda a, ax, kd: oracle.sum_axis(wrap(a) if isinstance(a, np.ndarray) else a, ax, kd),
        lambda o, a, s: oracle.unary(o, wrap(a) if isinstance(a, np.ndarray) else a, s),
        x, gamma, beta, eps)


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape", [[2, 3], [64, 100], [33, 1024], [8, 4096], [5, 16384], [3, 20000],
                                   [2, 3, 768], [17, 1]], ids=str)
def test_layer_norm_fused(shape, dtype):
    import oracle
    from tensorrs_b200 import device
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * 3 + 1.5).astype(dtype)
    F = shape[-1]
    gamma = rng.uniform(0.5, 1.5, [1, F]).astype(dtype)
    beta = rng.uniform(-0.5, 0.5, [1, F]).astype(dtype)
    eps = 1e-5
    dx, dg, db = contiguous(x), contiguous(gamma), contiguous(beta)
    got = to_host(device.layer_norm_lastdim(dx.view, dg.view, db.view, eps, empty(shape, dtype)))
    x2 = x.reshape(-1, F)
    ideal = _ideal_layer_norm(x2, gamma.reshape(-1), beta.reshape(-1), eps).reshape(shape)
    if dtype == np.float32:
        # f64 sums rounded once: the exactly-summed restatement, bit for bit,
        # except rows whose f64 sum rounds to the other f32 neighbour
        same = got == ideal
        rows_off = int((~same.reshape(-1, F)).any(axis=1).sum())
        assert rows_off <= max(1, x2.shape[0] // 100), f"{rows_off} rows differ from the exactly-summed restatement"
        assert np.allclose(got, ideal, rtol=1e-5, atol=1e-5 * float(np.abs(beta).max() + 1))
    else:
        # f64 sums in f64 (no wider type): F * 2^-53 relative on the sums
        assert np.allclose(got, ideal, rtol=F * 2.0**-50, atol=F * 2.0**-50)
    # against the reference's chain: its f32 sequential sums carry up to
    # (F-1) * 2^-24 relative error, amplified by 1/denom in x_hat
    ref = _chain_layer_norm(oracle.contiguous(x), oracle.contiguous(gamma), oracle.contiguous(beta), eps)
    tol = (F * np.finfo(dtype).eps * 4 + 1e-6) * (np.abs(ref) + np.abs(beta) + 1)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= tol)


def test_layer_norm_strided_input_and_gamma():
    """A transposed x (rows are storage columns) and gamma / beta given as [F]
    views with a stride."""
    from tensorrs_b200 import device
    rng = np.random.default_rng(9)
    st = rng.standard_normal(300 * 40).astype(np.float32)
    dx = DevView(st, [40, 300], [1, 40], 0)
    gst = rng.uniform(0.5, 1.5, 600).astype(np.float32)
    bst = rng.uniform(-0.5, 0.5, 600).astype(np.float32)
    dg = DevView(gst, [300], [2], 1)
    db = DevView(bst, [1, 300], [300, 2], 0)
    got = to_host(device.layer_norm_lastdim(dx.view, dg.view, db.view, 1e-5, empty([40, 300], np.float32)))
    x2 = np.ascontiguousarray(st.reshape(300, 40).T)
    ideal = _ideal_layer_norm(x2, gst[1::2].copy(), bst[0::2].copy(), 1e-5)
    assert np.allclose(got, ideal, rtol=1e-5, atol=1e-5)


def test_layer_norm_reference_properties():
    """nn/layer_norm.rs:145-199: a larger epsilon changes the output; the
    shapes (2x1, 2x4, 3x2 of consecutive numbers) are kept; a single feature
    normalises to 0."""
    from tensorrs_b200 import device
    x = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    dx = contiguous(x)
    g = contiguous(np.ones([1, 2], np.float32))
    b = contiguous(np.zeros([1, 2], np.float32))
    big = to_host(device.layer_norm_lastdim(dx.view, g.view, b.view, 1.0, empty([2, 2], np.float32)))
    small = to_host(device.layer_norm_lastdim(dx.view, g.view, b.view, 1e-8, empty([2, 2], np.float32)))
    assert np.abs(big - small).max() > 1e-6
    for batch, feats in [(2, 1), (2, 4), (3, 2)]:
        xs = np.arange(batch * feats, dtype=np.float32).reshape(batch, feats)
        out = to_host(device.layer_norm_lastdim(contiguous(xs).view, contiguous(np.ones([1, feats], np.float32)).view,
                                                contiguous(np.zeros([1, feats], np.float32)).view, 1e-5,
                                                empty([batch, feats], np.float32)))
        assert out.shape == (batch, feats)
        if feats == 1:
            assert np.array_equal(out, np.zeros_like(out))


def test_layer_norm_matches_the_chain_on_the_reference_known_answers():
    from _golden import check
    from conftest import golden_cases
    from tensorrs_b200 import device
    for case in [c for c in golden_cases() if c["op"] == "layer_norm"]:
        xs = [np.array(i["storage"], np.float32).reshape(i["shape"]) for i in case["inputs"]]
        ds = [contiguous(a) for a in xs]
        got = to_host(device.layer_norm_lastdim(ds[0].view, ds[1].view, ds[2].view, case["epsilon"],
                                                empty(xs[0].shape, np.float32)))
        check(case, got)
        import oracle
        ref = _chain_layer_norm(oracle.contiguous(xs[0]), oracle.contiguous(xs[1]), oracle.contiguous(xs[2]),
                                case["epsilon"])
        assert max_ulp(got, ref) <= 8, case["name"]
