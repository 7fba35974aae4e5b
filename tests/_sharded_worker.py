"""One rank of the several-GPU parity test (launched by torchrun, one process
per GPU; see test_sharded_gpu.py).

Every rank builds the same seeded global tensors, keeps its dim-0 shard on its
GPU, calls the trs_sharded_* entry points through the communicator, and checks
the global result it receives against the oracle run on the whole tensor:
integer sums, max and argmax bit-exact (NaN, tie and empty-shard rules
included), float sums within 1e-5 * sum|x| of the reference's sequential fold
and within 1 ulp + n * 2^-40 * sum|x| of the exact sum.  Each rank writes
<outdir>/rank<r>.json with its failures and exits non-zero if it has any.
"""
from __future__ import annotations

import datetime
import json
import os
import sys
import traceback
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def rand(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.standard_normal(size=shape).astype(dtype)
    return rng.integers(-1000, 1000, size=shape).astype(dtype)


def plant_specials(x: np.ndarray, counts: list[int]) -> None:
    """NaN / tie / -inf patterns whose answers depend on the cross-rank rules."""
    if x.dtype.kind != "f" or x.shape[0] < 4 or x.shape[1] < 9:
        return
    n = x.shape[0]
    x[0, 3] = np.nan                     # NaN at global index 0: sticky
    x[min(5, n - 1), 4] = np.nan         # NaN later: skipped
    x[:, 5] = 1.0                        # all equal: index 0
    offs = np.cumsum([0] + counts)
    hi = float(np.nanmax(x[:, 6])) + 1.0
    for r in range(1, len(counts)):      # the same maximum at the end of one shard and the start of the next
        if counts[r - 1] and counts[r]:
            x[offs[r] - 1, 6] = hi
            x[offs[r], 6] = hi
            break
    x[:, 7] = -np.inf                    # all -inf: index 0
    x[:, 8] = np.nan                     # all NaN: NaN, index 0
    x[n - 1, 8] = 2.0


def main(outdir: str) -> int:
    import torch
    import torch.distributed as dist

    import oracle
    from _util import assert_bit_exact
    from tensorrs_b200 import abi, device, sharding

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    lib = abi.load()
    comm = sharding.Communicator(lib, rank, world, dist, timeout_ms=60000)
    sh = torch.cuda.current_stream().cuda_stream
    failures: list[str] = []

    def run(name, fn):
        try:
            fn()
        except Exception:  # noqa: BLE001 -- every case reports, the run goes on
            failures.append(f"{name}: {traceback.format_exc(limit=3)}")

    def dev(a: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    def check_sum(got, ref, sabs, exact):
        got = np.asarray(got, np.float64)
        ref = np.asarray(ref, np.float64)
        assert got.shape == ref.shape, (got.shape, ref.shape)
        assert np.all(np.abs(got - ref) <= 1e-5 * sabs + 1e-30)
        assert np.all(np.abs(got - exact) <= np.abs(exact) * 2.0**-23 + 2.0**-40 * sabs + 1e-300)

    splits = {
        "even": lambda total: [sharding.shard_rows(total, world, r)[1] for r in range(world)],
        # rank r holds about (r + 1) / sum(1..world) of the rows
        "ragged": lambda total: [total * (r + 1) // (world * (world + 1) // 2) for r in range(world - 1)],
        "rank0_empty": lambda total: [0] + [total // max(1, world - 1)] * (world - 1),
    }

    def counts_for(kind, total):
        c = splits[kind](total)
        if kind == "ragged":
            c = c + [total - sum(c)]
        if kind == "rank0_empty":
            c[-1] += total - sum(c)
        assert sum(c) == total and min(c) >= 0
        return c

    for dtype in (np.float32, np.float64, np.int32, np.int64):
        for kind in ("even", "ragged", "rank0_empty"):
            for total, width in ((64, 33), (1031, 1000), (4096, 2048)):
                name = f"axis0 {np.dtype(dtype).name} {kind} [{total},{width}]"
                counts = counts_for(kind, total)
                offs = sharding.row_offsets(counts)
                x = rand((total, width), dtype, total + width + len(name))
                plant_specials(x, counts)
                mine = x[offs[rank]:offs[rank] + counts[rank]]
                t = dev(mine)
                xv = oracle.contiguous(x)

                def case_sum(t=t, x=x, xv=xv, width=width, dtype=dtype):
                    out = torch.empty((width,), dtype=t.dtype, device="cuda")
                    comm.sum_axis0(device.view_of(t), device.view_of(out), sh)
                    torch.cuda.synchronize()
                    got = out.cpu().numpy()
                    ref = oracle.sum_axis(xv, 0, False)
                    if np.dtype(dtype).kind == "i":
                        assert_bit_exact(got, ref, "sum_axis0")
                    else:
                        xd = np.where(np.isfinite(x), x, 0).astype(np.float64)
                        fin = np.all(np.isfinite(x), axis=0)
                        check_sum(got[fin], ref[fin], np.abs(xd).sum(0)[fin], xd.sum(0)[fin])
                        assert_bit_exact(got[~fin], ref[~fin], "sum_axis0 of non-finite columns")

                def case_max(t=t, xv=xv, width=width):
                    mx = torch.empty((width,), dtype=t.dtype, device="cuda")
                    am = torch.empty((width,), dtype=torch.int64, device="cuda")
                    comm.max_axis0(device.view_of(t), device.view_of(mx), sh)
                    comm.argmax_axis0(device.view_of(t), device.view_of(am), sh)
                    torch.cuda.synchronize()
                    rmx, ram = oracle.max_argmax_axis(xv, 0)
                    assert_bit_exact(mx.cpu().numpy(), rmx, "max_axis0")
                    assert_bit_exact(am.cpu().numpy(), ram.astype(np.int64), "argmax_axis0")

                run(name + " sum", case_sum)
                run(name + " max/argmax", case_max)

    # full sum and the fused element-wise + sum (the sharded bench step)
    for dtype in (np.float32, np.int32):
        total, width = 2000, 1536
        counts = counts_for("ragged", total)
        offs = sharding.row_offsets(counts)
        x = rand((total, width), dtype, 77)
        mine = x[offs[rank]:offs[rank] + counts[rank]]

        def case_full(mine=mine, x=x, dtype=dtype):
            t = dev(mine)
            out = torch.empty((1,), dtype=t.dtype, device="cuda")
            comm.sum(device.view_of(t), device.view_of(out), sh)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            ref = np.asarray(oracle.sum_all(oracle.contiguous(x))).reshape(1)
            if np.dtype(dtype).kind == "i":
                assert_bit_exact(got, ref.astype(dtype), "sharded sum")
            else:
                xd = x.astype(np.float64)
                check_sum(got, ref, np.abs(xd).sum(), np.array([xd.sum()]))

        run(f"sum {np.dtype(dtype).name}", case_full)

    def case_fma():
        total, width = 4097, 2048
        counts = counts_for("ragged", total)
        offs = sharding.row_offsets(counts)
        a = oracle.fill_uniform(np.float32, total * width, 4).reshape(total, width)
        b = oracle.fill_uniform(np.float32, total * width, 5).reshape(total, width)
        c = oracle.fill_uniform(np.float32, width, 6)
        lo, n = offs[rank], counts[rank]
        ta, tb, tc = dev(a[lo:lo + n]), dev(b[lo:lo + n]), dev(c)
        ty = torch.empty((n, width), dtype=torch.float32, device="cuda")
        ts = torch.empty((1,), dtype=torch.float32, device="cuda")
        prog = abi.program(3, abi.MUL, abi.ADD)
        comm.elementwise_sum(prog, [device.view_of(ta), device.view_of(tb), device.view_of(tc)],
                             device.view_of(ty), device.view_of(ts), sh)
        torch.cuda.synchronize()
        y_ref = oracle.program(3, "mul", "add", "none",
                               [oracle.contiguous(a), oracle.contiguous(b), oracle.contiguous(c)])
        assert_bit_exact(ty.cpu().numpy(), y_ref[lo:lo + n], "Y shard")
        s_ref = np.asarray(oracle.sum_all(oracle.contiguous(y_ref))).reshape(1)
        yd = y_ref.astype(np.float64)
        check_sum(ts.cpu().numpy(), s_ref, np.abs(yd).sum(), np.array([yd.sum()]))

    run("elementwise_sum fma", case_fma)

    # the combine of the full sums: over NVLink peer memory when every rank
    # mapped every peer's slot buffer; many calls in a row (the slot sets
    # alternate with the call's parity), then the same sums through a
    # communicator forced onto ncclAllReduce, which must agree
    exchange = comm.peer_exchange
    xs = [rand((257 + 31 * i, 129), np.float32 if i % 2 else np.int64, 500 + i) for i in range(40)]

    def sums_through(c):
        got = []
        for x in xs:
            counts = counts_for("ragged", x.shape[0])
            offs = sharding.row_offsets(counts)
            t = dev(x[offs[rank]:offs[rank] + counts[rank]])
            out = torch.empty((1,), dtype=t.dtype, device="cuda")
            c.sum(device.view_of(t), device.view_of(out), sh)
            got.append(out)
        torch.cuda.synchronize()
        return [o.cpu().numpy() for o in got]

    def case_many():
        got = sums_through(comm)
        for x, g in zip(xs, got):
            ref = np.asarray(oracle.sum_all(oracle.contiguous(x))).reshape(1)
            if x.dtype.kind == "i":
                assert_bit_exact(g, ref.astype(x.dtype), "sum in a row of calls")
            else:
                xd = x.astype(np.float64)
                check_sum(g, ref, np.abs(xd).sum(), np.array([xd.sum()]))
        os.environ["TRS_PEER_EXCHANGE"] = "0"
        try:
            nc = sharding.Communicator(lib, rank, world, dist, timeout_ms=60000)
        finally:
            del os.environ["TRS_PEER_EXCHANGE"]
        try:
            assert not nc.peer_exchange
            via_nccl = sums_through(nc)
        finally:
            nc.destroy()
        for x, g, h in zip(xs, got, via_nccl):
            if x.dtype.kind == "i":
                assert_bit_exact(g, h, "exchange vs NCCL")
            else:  # both f64 sums of `world` partials rounded once
                assert abs(float(g[0]) - float(h[0])) <= float(np.spacing(np.float32(abs(h[0]))))

    run("sums in a row, exchange vs NCCL", case_many)

    def case_axis0_many():
        """Six axis-0 reductions in a row (each arena parity three times) through
        the exchange and through a communicator forced onto NCCL: max and argmax
        identical, sums within one ulp of each other (both the f64 sum of the
        ranks' partials, rounded once)."""
        data = []
        for j, (total, width) in enumerate([(64, 33), (1031, 1000), (4096, 2048)] * 2):
            counts = counts_for("ragged", total)
            offs = sharding.row_offsets(counts)
            x = rand((total, width), np.float32, 500 + j)
            data.append((dev(x[offs[rank]:offs[rank] + counts[rank]]), width))

        def through(c):
            res = []
            for t, width in data:
                s_ = torch.empty((width,), dtype=t.dtype, device="cuda")
                m_ = torch.empty((width,), dtype=t.dtype, device="cuda")
                a_ = torch.empty((width,), dtype=torch.int64, device="cuda")
                c.sum_axis0(device.view_of(t), device.view_of(s_), sh)
                c.max_axis0(device.view_of(t), device.view_of(m_), sh)
                c.argmax_axis0(device.view_of(t), device.view_of(a_), sh)
                res.append((s_, m_, a_))
            torch.cuda.synchronize()
            return [tuple(v.cpu().numpy() for v in r) for r in res]

        got = through(comm)
        os.environ["TRS_PEER_EXCHANGE"] = "0"
        try:
            nc = sharding.Communicator(lib, rank, world, dist, timeout_ms=60000)
        finally:
            del os.environ["TRS_PEER_EXCHANGE"]
        try:
            assert not nc.peer_exchange
            ref = through(nc)
        finally:
            nc.destroy()
        for (gs, gm, ga), (rs, rm, ra) in zip(got, ref):
            assert_bit_exact(gm, rm, "max_axis0, exchange vs NCCL")
            assert_bit_exact(ga, ra, "argmax_axis0, exchange vs NCCL")
            assert np.all(np.abs(gs.astype(np.float64) - rs.astype(np.float64)) <= np.spacing(np.abs(rs)))

    run("axis-0 reductions in a row, exchange vs NCCL", case_axis0_many)

    def case_peer_timeout():
        """Rank 0 makes a sharded sum that rank 1 skips: its kernel's wait for
        rank 1's partial runs out (about 2 s), it reports bit 1 of the
        async-error word and writes NaN; rank 1 keeps its buffers alive until
        rank 0's kernel has ended (the barrier), then both destroy the
        communicator, whose calls are no longer matched."""
        import time
        tc = sharding.Communicator(lib, rank, world, dist, timeout_ms=60000)
        try:
            if not tc.peer_exchange:
                return
            if rank == 0:
                t = dev(np.ones((8, 8), np.float32))
                out = torch.zeros((1,), dtype=torch.float32, device="cuda")
                t0 = time.monotonic()
                tc.sum(device.view_of(t), device.view_of(out), sh)
                torch.cuda.synchronize()
                waited = time.monotonic() - t0
                code = ctypes_async_error(lib)
                assert code & 2, f"async-error word {code}, waited {waited:.2f} s"
                assert np.isnan(out.cpu().numpy()[0])
                assert 0.5 <= waited <= 60, waited
                # the same for an axis-0 sum: its combine waits on the
                # exchange's flags, runs out, and writes NaN
                cols = torch.zeros((8,), dtype=torch.float32, device="cuda")
                tc.sum_axis0(device.view_of(t), device.view_of(cols), sh)
                torch.cuda.synchronize()
                code = ctypes_async_error(lib)
                assert code & 2, f"axis-0 sum: async-error word {code}"
                assert np.isnan(cols.cpu().numpy()).all()
            dist.barrier()
        finally:
            tc.destroy()

    if world == 2:
        run("peer exchange wait runs out", case_peer_timeout)

    err = ctypes_async_error(lib)
    if err:
        failures.append(f"async error word {err}")
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()
    Path(outdir, f"rank{rank}.json").write_text(json.dumps({"rank": rank, "world": world, "failures": failures,
                                                           "peer_exchange": exchange}))
    return 1 if failures else 0


def ctypes_async_error(lib) -> int:
    import ctypes
    v = ctypes.c_int32(0)
    lib.trs_async_error(ctypes.byref(v))
    return int(v.value)


if __name__ == "__main__":
    sys.exit(main(sys.argv[1]))
