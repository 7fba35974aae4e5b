"""trs_sum_noalloc: the full sum for callers that cannot allocate device
memory while they run -- a host that hands all device memory to its own arena
at start-up, or a code path that must not enter the CUDA allocator.  Its
partial sums live in a static device array instead of pool scratch.

Checked here: it makes no scratch allocation (the library's allocation
counter does not move across it), its result equals trs_sum's and lies within
the sum tolerance of the oracle's (the reference's sequential fold, and the
exact sum) on two different inputs in a row, an empty input sums to 0, and a
sum needing more partials than the array holds is refused before any launch.

This file is collected last, so a run that stops at its first failure has run
every other test before it; it also passes alone in a fresh process (its first
call then performs the per-device set-up)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _gpu import contiguous

pytestmark = pytest.mark.gpu


def _sum_noalloc(x_view, dtype):
    """trs_sum_noalloc of the view; asserts it allocated no scratch."""
    import torch

    from tensorrs_b200 import abi, device
    lib = abi.load()
    out = torch.full((1,), 7, dtype=dtype, device="cuda")
    before = lib.trs_scratch_alloc_count()
    abi.check(lib.trs_sum_noalloc(ctypes.byref(x_view), ctypes.byref(device.view_of(out)), device.stream_handle()))
    assert lib.trs_scratch_alloc_count() == before, "trs_sum_noalloc allocated scratch"
    torch.cuda.synchronize()
    return out.cpu().numpy()[0]


def _sum_pool(x_view, dtype):
    import torch

    from tensorrs_b200 import abi, device
    out = torch.empty((1,), dtype=dtype, device="cuda")
    abi.check(abi.load().trs_sum(ctypes.byref(x_view), ctypes.byref(device.view_of(out)), device.stream_handle()))
    torch.cuda.synchronize()
    return out.cpu().numpy()[0]


def test_no_alloc_sum_matches_trs_sum_and_the_oracle_on_two_calls_in_a_row():
    import torch

    import oracle
    # two different inputs back to back: the second call must not see the
    # first call's partials (the no-alloc calls come first)
    xs = [oracle.fill_uniform(np.float32, 4096 * 8192, 4).reshape(4096, 8192),
          oracle.fill_normal(np.float32, 1000 * 1003, 5).reshape(1000, 1003)]
    dev = [contiguous(x) for x in xs]
    got = [_sum_noalloc(d.view, torch.float32) for d in dev]
    for x, d, g in zip(xs, dev, got):
        exact, sabs = oracle.sum_f64(d.host_view())
        fold = float(oracle.sum_all(d.host_view()))
        # the tolerance of every sum test: 1e-5 * sum|x| of the reference's
        # sequential f32 fold, and the f64-accumulation bound of the exact sum
        assert abs(float(g) - fold) <= 1e-5 * sabs
        assert abs(float(g) - exact) <= abs(exact) * 2.0**-23 + 2.0**-40 * sabs
        # the same kernels in the same order as trs_sum: the same bits
        assert g == _sum_pool(d.view, torch.float32)


def test_no_alloc_sum_on_a_strided_view_and_integers():
    import torch

    from tensorrs_b200 import device
    z = torch.arange(0, 300 * 700, dtype=torch.int64, device="cuda").reshape(300, 700)
    zt = device.view_of(z, [700, 300], [1, 700], 0)
    got = _sum_noalloc(zt, torch.int64)
    assert got == _sum_pool(zt, torch.int64) == np.int64(300 * 700 * (300 * 700 - 1) // 2)


def test_no_alloc_sum_of_an_empty_tensor_is_zero():
    import torch

    from tensorrs_b200 import device
    for shape in ([0], [3, 0]):
        e = torch.empty(shape, dtype=torch.float32, device="cuda")
        got = _sum_noalloc(device.view_of(e), torch.float32)
        assert got == 0.0 and not np.signbit(got)


def test_no_alloc_sum_refuses_more_partials_than_its_array_holds():
    """A [1024, 2^30] broadcast view of 1024 elements (stride 0 along the
    rows) needs far more than 8192 per-block partials; the call fails with
    TRS_ERR_ARG before launching anything."""
    import torch

    from tensorrs_b200 import abi, device
    lib = abi.load()
    base = torch.ones(1024, dtype=torch.float32, device="cuda")
    big = device.view_of(base, [1024, 1 << 30], [1, 0], 0)
    out = torch.zeros((1,), dtype=torch.float32, device="cuda")
    launches, allocs = lib.trs_launch_count(), lib.trs_scratch_alloc_count()
    st = lib.trs_sum_noalloc(ctypes.byref(big), ctypes.byref(device.view_of(out)), device.stream_handle())
    assert st == abi.ERR_ARG
    assert "partials" in abi.last_error()
    assert lib.trs_launch_count() == launches and lib.trs_scratch_alloc_count() == allocs
    # the array is still usable afterwards
    small = contiguous(np.arange(10, dtype=np.float32))
    assert _sum_noalloc(small.view, torch.float32) == 45.0
