"""Several-rank host logic on CPU: two `gloo` ranks (world_size 2) run the
host side of the sharded path without a GPU.

* `shard_rows` / `row_offsets` split rows into contiguous runs that cover the
  tensor, ranks with zero rows included;
* `exchange_unique_id` hands every rank rank 0's 128-byte id;
* the combine rules the sharded kernels implement reproduce the reference on
  the unsplit tensor: per-rank (largest non-NaN value, its first global
  index) records folded in rank order, the first element of the lowest
  non-empty rank standing in for global index 0 (a NaN there is sticky, as in
  max_axis, base.rs:1404-1411), and per-rank f64 partial sums all-reduced then
  rounded once.  The oracle on the whole tensor is the checker.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _records(shard: np.ndarray, base: int):
    """Per-column (value, global index) of the largest non-NaN element (first
    index on ties); index -1 when the shard has none."""
    rows, w = shard.shape
    vals = np.zeros(w, shard.dtype)
    idx = np.full(w, -1, np.int64)
    for j in range(w):
        col = shard[:, j]
        ok = ~np.isnan(col) if col.dtype.kind == "f" else np.ones(rows, bool)
        if ok.any():
            k = int(np.flatnonzero(ok)[np.argmax(col[ok])])
            vals[j], idx[j] = col[k], base + k
    return vals, idx


def _combine(all_vals, all_idx, first_row):
    w = all_vals[0].shape[0]
    out_v = np.zeros(w, all_vals[0].dtype)
    out_i = np.full(w, -1, np.int64)
    for v, i in zip(all_vals, all_idx):
        take = (i >= 0) & ((out_i < 0) | (v > out_v))
        out_v = np.where(take, v, out_v)
        out_i = np.where(take, i, out_i)
    fix = np.isnan(first_row) | (out_i < 0) if first_row.dtype.kind == "f" else out_i < 0
    return np.where(fix, first_row, out_v), np.where(fix, 0, out_i)


def _rank_main(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import oracle
    from tensorrs_b200 import sharding
    errors = []
    try:
        # splits
        for total in (0, 1, 7, 64, 1031):
            first, rows = sharding.shard_rows(total, world, rank)
            got = [None] * world
            dist.all_gather_object(got, (first, rows))
            assert got[0][0] == 0 and sum(r for _, r in got) == total
            assert all(got[k][0] + got[k][1] == got[k + 1][0] for k in range(world - 1))
            assert sharding.row_offsets([r for _, r in got]) == [f for f, _ in got]
        # id exchange
        rng = np.random.default_rng(1234)
        uid = sharding.exchange_unique_id(lambda: rng.integers(0, 256, 128, dtype=np.uint8).tobytes(), rank, dist)
        ids = [None] * world
        dist.all_gather_object(ids, uid)
        assert all(i == ids[0] for i in ids) and len(uid) == 128
        # combine rules against the oracle on the unsplit tensor
        for dtype in (np.float32, np.float64, np.int32):
            for counts in ([0, 40], [1, 39], [23, 17], [40, 0]):
                total, w = sum(counts), 11
                g = np.random.default_rng(total + w)
                x = (g.standard_normal((total, w)) if np.dtype(dtype).kind == "f"
                     else g.integers(-5, 5, (total, w))).astype(dtype)
                if x.dtype.kind == "f":
                    x[0, 0] = np.nan
                    x[3, 1] = np.nan
                    x[:, 2] = 0.5
                    x[:, 3] = -np.inf
                    x[:, 4] = np.nan
                    x[-1, 4] = 1.0
                    x[counts[0] - 1 if counts[0] else 0, 5] = 9.0
                    x[min(counts[0], total - 1), 5] = 9.0
                offs = sharding.row_offsets(counts)
                mine = x[offs[rank]:offs[rank] + counts[rank]]
                v, i = _records(mine, offs[rank])
                all_v, all_i = [None] * world, [None] * world
                dist.all_gather_object(all_v, v)
                dist.all_gather_object(all_i, i)
                first_rank = next(k for k in range(world) if counts[k] > 0)
                fr = [None] * world
                dist.all_gather_object(fr, mine[0] if counts[rank] else None)
                mv, mi = _combine(all_v, all_i, fr[first_rank])
                rv, ri = oracle.max_argmax_axis(oracle.contiguous(x), 0)
                assert np.array_equal(mi, ri), (dtype, counts, mi, ri)
                assert np.array_equal(np.isnan(mv) if x.dtype.kind == "f" else mv,
                                      np.isnan(rv) if x.dtype.kind == "f" else rv)
                if x.dtype.kind == "f":
                    ok = ~np.isnan(rv)
                    assert np.array_equal(mv[ok], rv[ok])
                # sums: f64 partials all-reduced, rounded once
                if x.dtype.kind == "f":
                    part = torch.from_numpy(mine.astype(np.float64).sum(axis=0) if counts[rank]
                                            else np.zeros(w))
                    dist.all_reduce(part)
                    s = part.numpy().astype(dtype)
                    ref = oracle.sum_axis(oracle.contiguous(x), 0, False)
                    fin = np.all(np.isfinite(x), axis=0)
                    sabs = np.abs(np.where(np.isfinite(x), x, 0).astype(np.float64)).sum(0)
                    assert np.all(np.abs(s[fin].astype(np.float64) - ref[fin]) <= 1e-5 * sabs[fin] + 1e-30)
    except Exception as e:  # noqa: BLE001
        import traceback
        errors.append(f"rank {rank}: {e!r}\n{traceback.format_exc(limit=4)}")
    results[rank] = errors
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_split_exchange_and_combine():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert set(results.keys()) == {0, 1}
    assert results[0] == [] and results[1] == [], dict(results)
