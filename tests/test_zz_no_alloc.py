"""trs_sum_noalloc: the full sum for callers that cannot allocate device
memory while they run (a host owning all device memory through its own arena,
or a path that must not enter the CUDA allocator).  Its partial sums live in a
static device array instead of pool scratch.

This file is collected last, so a run that stops at its first failure has run
every other test before it; it also passes alone in a fresh process (its first
call then performs the per-device set-up)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sum_both(x_view, dtype):
    import torch

    from tensorrs_b200 import abi, device
    lib = abi.load()
    a = torch.empty((1,), dtype=dtype, device="cuda")
    b = torch.empty((1,), dtype=dtype, device="cuda")
    sh = device.stream_handle()
    abi.check(lib.trs_sum(ctypes.byref(x_view), ctypes.byref(device.view_of(a)), sh))
    abi.check(lib.trs_sum_noalloc(ctypes.byref(x_view), ctypes.byref(device.view_of(b)), sh))
    torch.cuda.synchronize()
    return a.cpu().numpy()[0], b.cpu().numpy()[0]


def test_no_alloc_sum_matches_trs_sum_on_two_calls_in_a_row():
    import torch

    from tensorrs_b200 import device
    # two different inputs back to back: the second call must not see the
    # first call's partials
    x = device.fill_uniform(torch.empty((4096, 8192), dtype=torch.float32, device="cuda"), 4)
    y = device.fill_normal(torch.empty((1000, 1003), dtype=torch.float32, device="cuda"), 5)
    for t in (x, y):
        want, got = _sum_both(device.view_of(t), torch.float32)
        # the same kernels in the same order: identical, within the sum
        # tolerance the other tests use (1e-5 of the sum of magnitudes)
        sabs = float(t.abs().double().sum())
        assert abs(float(got) - float(want)) <= 1e-5 * sabs
        assert got == want


def test_no_alloc_sum_on_a_strided_view_and_integers():
    import torch

    from tensorrs_b200 import device
    z = torch.arange(0, 300 * 700, dtype=torch.int64, device="cuda").reshape(300, 700)
    zt = device.view_of(z, [700, 300], [1, 700], 0)
    want, got = _sum_both(zt, torch.int64)
    assert got == want == np.int64(300 * 700 * (300 * 700 - 1) // 2)
