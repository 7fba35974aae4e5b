"""The oracle's optimiser steps (SGD, RMSprop, Adam for one parameter; the
reference has no unit test with known values for them) pinned against an
independent restatement of the reference's chain of tensor calls in numpy
scalar arithmetic: every numpy f32/f64 operation is one IEEE operation
rounded to nearest-even, as each of the reference's calls is; sqrt is
correctly rounded in both; beta^t is glibc's powf / pow called through
ctypes (what the reference's std calls; numpy's own float32 power differs
from powf in the last bit for some arguments)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

_libm = ctypes.CDLL("libm.so.6")
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
_libm.pow.restype = ctypes.c_double
_libm.pow.argtypes = [ctypes.c_double, ctypes.c_double]


def _pow(T, b, t):
    return T(_libm.powf(b, t)) if T is np.float32 else T(_libm.pow(b, t))


def _numpy_step(kind, p, g, m, v, lr, b1, b2, eps, t):
    T = p.dtype.type
    lr, b1, b2, eps = T(lr), T(b1), T(b2), T(eps)
    one = T(1)
    if kind == "sgd":                                   # optim/sgd.rs:35
        return p - g * lr, m, v
    if kind == "rmsprop":                               # optim/rmsprop.rs:36-44 (alpha in b2)
        v = v * b2 + (g * g) * (one - b2)
        return p - (g * lr) / (np.sqrt(v) + eps), m, v
    m = m * b1 + g * (one - b1)                         # optim/adam.rs:128-142
    v = v * b2 + (g * g) * (one - b2)
    tt = T(t)
    mh = m / (one - _pow(T, b1, tt))
    vh = v / (one - _pow(T, b2, tt))
    return p - (mh * lr) / (np.sqrt(vh) + eps), m, v


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("kind", ["sgd", "rmsprop", "adam"])
def test_oracle_optimiser_steps_equal_the_reference_chain(kind, dtype):
    import oracle
    rng = np.random.default_rng(5)
    n = 10007
    p = rng.standard_normal(n).astype(dtype)
    m = np.zeros(n, dtype)
    v = np.zeros(n, dtype)
    P, M, W = p.copy(), m.copy(), v.copy()
    b2 = 0.99 if kind == "rmsprop" else 0.999
    for t in range(1, 5):
        with np.errstate(over="ignore", invalid="ignore"):
            g = (rng.standard_normal(n) * 0.1).astype(dtype)
            g[:4] = [0.0, -0.0, 1e-30, -1e30]
            oracle.opt_step(kind, p, g, m if kind == "adam" else None, v if kind != "sgd" else None, 0.01,
                            0.9, b2, 1e-8, t)
            P, M, W = _numpy_step(kind, P, g, M, W, 0.01, 0.9, b2, 1e-8, t)
            assert np.array_equal(p.view(np.uint8), P.view(np.uint8)), (kind, t)
            if kind == "adam":
                assert np.array_equal(m, M)
            if kind != "sgd":
                assert np.array_equal(v, W)


def test_oracle_adam_first_step_known_value():
    """At t = 1 with m = v = 0, Adam moves every weight by lr * g / (|g| + eps')
    where the bias corrections cancel (1 - b) exactly: for g = 0.5 and
    lr = 0.1 the f32 chain gives 1 - 0.1 = 0.9 (0.100000024 * 0.5 / 0.100000024)."""
    import oracle
    p = np.ones(3, np.float32)
    g = np.full(3, 0.5, np.float32)
    m = np.zeros(3, np.float32)
    v = np.zeros(3, np.float32)
    oracle.opt_step("adam", p, g, m, v, 0.1, t=1)
    assert np.all(np.abs(p - 0.9) < 1e-6)
