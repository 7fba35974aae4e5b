"""Benchmark of the broadcast-elementwise / full-reduction hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl trs|reference]
    python bench.py --suite      # every kernel of the path on its configuration

Default workload (the sharded configuration, run at 1/2/4/8 GPUs):
    Y = A & B + c, s = sum(Y)  with A, B f32 [65536, 32768] ~ U(-1,1) (8 GiB
    each), c f32 [32768] ~ U(-1,1), seed 4; A and B split on dim 0 across the
    ranks (strong scaling: the total problem is fixed), the sum combined with
    one NCCL all-reduce of f64 partials.
A step is one fused pass through the C ABI (trs_elementwise_sum, or
trs_sharded_elementwise_sum for N > 1): Y written, sum(Y) returned.

The metric is achieved HBM bandwidth: algorithmic bytes (every tensor read
once at its stored size, every output written once) / time, whole job.
`value` times device-resident inputs with CUDA events (max over ranks);
`e2e` times the same call with host buffers, the host->device copies of A, B
and c and the device->host read of the sum inside the timed region.  Inputs
(8 GiB per operand) exceed the 126 MB L2, so no flush is needed.

--impl reference times the reference's own CPU algorithm (its restatement in
oracle/, with all host threads) on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 65536, 32768
SEED_A, SEED_B, SEED_C = 4, 5, 6


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="trs", choices=["trs", "reference"])
    ap.add_argument("--workload", default="fma_sum")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="global rows of A and B (default 65536; smaller only for profiler captures)")
    ap.add_argument("--suite", action="store_true",
                    help="time every kernel of the path on its configuration (one JSON line each)")
    ap.add_argument("--only", default=None,
                    help="with --suite: only the entries whose 'config: kernel' name contains this text")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_bytes(rows: int, cols: int, ranks: int) -> int:
    """Algorithmic bytes of one step: A and B read, Y written (4 B each), c read
    by every rank, the one-element sum written."""
    return 3 * 4 * rows * cols + ranks * 4 * cols + 4


# ---------------------------------------------------------------------------
# CPU side: the reference's algorithm (oracle restatement), bounded sample
# ---------------------------------------------------------------------------
def cpu_reference_sample(seconds: float, threads: int) -> dict:
    """Times `&(&a & &b) + &c` then `.sum()` exactly as the reference runs them
    (binary_op fast path for a & b, broadcast path with storage_indices for
    + c, packed_data + serial fold for sum) on a row sample of the workload."""
    import oracle
    oracle.set_threads(threads)
    rows = 512
    a = oracle.fill_uniform(np.float32, rows * COLS, SEED_A)
    b = oracle.fill_uniform(np.float32, rows * COLS, SEED_B)
    c = oracle.fill_uniform(np.float32, COLS, SEED_C)
    av = oracle.HostView(a, [rows, COLS])
    bv = oracle.HostView(b, [rows, COLS])
    cv = oracle.HostView(c, [COLS])
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        t = oracle.binary("mul", av, bv)
        y = oracle.binary("add", oracle.HostView(t.reshape(-1), [rows, COLS]), cv)
        oracle.sum_all(oracle.HostView(y.reshape(-1), [rows, COLS]))
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 2:
            break
    sec = float(np.median(times))
    nbytes = workload_bytes(rows, COLS, 1)
    return {
        "value": round(nbytes / sec / 1e9, 3), "unit": "GB/s", "cores": threads,
        "kind": "port",
        "sample": f"{rows} of {ROWS} rows ([{rows},{COLS}] f32), {len(times)} timed passes, median "
                  f"{sec * 1e3:.1f} ms/pass; C++ restatement of binary_op/storage_indices/sum "
                  f"(oracle/oracle.cpp) on {threads} OpenMP threads",
        "ms_per_pass": round(sec * 1e3, 3),
    }


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    base = cpu_reference_sample(max(2.0, min(args.cpu_seconds, 30.0)), threads)
    line = {
        "impl": "reference", "metric": "achieved HBM GB/s (fraction of 8 TB/s) for broadcast-elementwise & axis-reduce",
        "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": base["ms_per_pass"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded splitmix64 uniforms)",
        "config": {"workload": "fma_sum: Y = A & B + c, sum(Y); A,B f32 [65536,32768], c [32768]; seed 4",
                   "timed": "row sample on host cores"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def ncu_traffic(workload: str, rows: int):
    """DRAM bytes (read + write) per launch of the dominant kernel, from the
    committed ncu capture summary, scaled from the captured row count to this
    launch's rows (the traffic of this streaming kernel grows in proportion)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        rec = json.loads(p.read_text()).get(workload)
    except ValueError:
        return None
    if not rec:
        return None
    return int(rec["dram_bytes_per_launch"] * rows / rec["rows"])


def run_trs(args) -> None:
    import torch

    from tensorrs_b200 import abi, device

    rank, world, local = dist_env()
    if args.workload != "fma_sum":
        raise SystemExit("only the fma_sum workload is a bench line; the others are parity cases")
    torch.cuda.set_device(local)
    lib = abi.load()
    dist = None
    comm = ctypes.c_void_p()
    if world > 1:
        import datetime

        import torch.distributed as dist
        from tensorrs_b200 import sharding
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        communicator = sharding.Communicator(lib, rank, world, dist, timeout_ms=120000)
        comm = communicator.handle

    total_rows = args.rows
    assert total_rows % world == 0
    rows = total_rows // world
    r0 = rank * rows
    f32 = torch.float32
    A = torch.empty((rows, COLS), dtype=f32, device="cuda")
    B = torch.empty((rows, COLS), dtype=f32, device="cuda")
    C = torch.empty((COLS,), dtype=f32, device="cuda")
    Y = torch.empty((rows, COLS), dtype=f32, device="cuda")
    S = torch.empty((1,), dtype=f32, device="cuda")
    device.fill_uniform(A, SEED_A, first=r0 * COLS)
    device.fill_uniform(B, SEED_B, first=r0 * COLS)
    device.fill_uniform(C, SEED_C)
    torch.cuda.synchronize()

    prog = abi.program(3, abi.MUL, abi.ADD)
    ins = abi.views_array([device.view_of(A), device.view_of(B), device.view_of(C)])
    yv, sv = device.view_of(Y), device.view_of(S)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    def step():
        if world > 1:
            st = lib.trs_sharded_elementwise_sum(comm, ctypes.byref(prog), ins, ctypes.byref(yv), ctypes.byref(sv), sh)
        else:
            st = lib.trs_elementwise_sum(ctypes.byref(prog), ins, ctypes.byref(yv), ctypes.byref(sv), sh)
        abi.check(st)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    launches0 = lib.trs_launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    t_end.record(stream)
    barrier()
    launches = lib.trs_launch_count() - launches0
    clk = clocks.stop()
    ms_total = t_start.elapsed_time(t_end)
    per_call_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))

    ms_step = ms_total / args.steps
    if dist is not None:
        t = torch.tensor([ms_step, per_call_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step, per_call_ms = float(t[0]), float(t[1])

    s_val = float(S.cpu()[0])

    total_bytes = workload_bytes(total_rows, COLS, world)
    value = total_bytes / (ms_step * 1e-3) / 1e9
    # roofline of the dominant kernel on one GPU: bytes one launch moves / its duration
    bytes_per_launch = workload_bytes(rows, COLS, 1)
    achieved = bytes_per_launch / (per_call_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    traffic = ncu_traffic("fma_sum", rows)

    # e2e: the same call from host buffers (pinned), copies inside the timed region
    e2e = None
    if args.e2e_steps > 0:
        hA = torch.empty((rows, COLS), dtype=f32, pin_memory=True)
        hB = torch.empty((rows, COLS), dtype=f32, pin_memory=True)
        hC = torch.empty((COLS,), dtype=f32, pin_memory=True)
        hS = torch.empty((1,), dtype=f32, pin_memory=True)
        hA.copy_(A)
        hB.copy_(B)
        hC.copy_(C)
        barrier()
        nA = hA.numel() * 4
        nC = hC.numel() * 4

        def e2e_step():
            abi.check(lib.trs_memcpy_htod(A.data_ptr(), hA.data_ptr(), nA, sh))
            abi.check(lib.trs_memcpy_htod(B.data_ptr(), hB.data_ptr(), nA, sh))
            abi.check(lib.trs_memcpy_htod(C.data_ptr(), hC.data_ptr(), nC, sh))
            step()
            abi.check(lib.trs_memcpy_dtoh(hS.data_ptr(), S.data_ptr(), 4, sh))
            abi.check(lib.trs_stream_synchronize(sh))

        e2e_step()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e_ms = e0.elapsed_time(e1) / args.e2e_steps
        if dist is not None:
            t = torch.tensor([e_ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t[0])
        e2e = {"value": round(total_bytes / (e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": 2 * nA + nC, "d2h_bytes_per_step": 4, "ms_per_step": round(e_ms, 3),
               "note": "A, B, c copied host->device and sum(Y) device->host each step through trs_memcpy_*; "
                       "PCIe-bound"}
        del hA, hB

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_sample(args.cpu_seconds, os.cpu_count() or 1)
        cpu.pop("ms_per_pass", None)

    if rank == 0:
        line = {
            "metric": "achieved HBM GB/s (fraction of 8 TB/s) for broadcast-elementwise & axis-reduce",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded splitmix64 uniforms generated on device)",
            "config": {"workload": f"fma_sum: Y = A & B + c and sum(Y) (config 5); A,B f32 [{total_rows},32768] "
                                   "~U(-1,1) split on dim 0, c f32 [32768], seed 4",
                       "global_rows": total_rows, "cols": COLS, "rows_per_gpu": rows,
                       "bytes_per_step": total_bytes, "l2": "inputs 8 GiB/operand >> 126 MB L2, no flush",
                       "parallelism": f"dim-0 shards x{world}" + (", NCCL all-reduce of f64 partials" if world > 1 else "")},
            "elements_per_s": round(total_rows * COLS / (ms_step * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "ew_stream_kernel<float, MulAdd, 3 bulk inputs, write, sum> + sum_finalize_kernel "
                                   "(one trs_elementwise_sum call; the finalize is ~2 us of the step)",
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "clocks": clk,
            "gpu_launches": int(launches),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "sum": s_val,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        communicator.destroy()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# --suite: every kernel of the path on its configuration, one JSON line each
# ---------------------------------------------------------------------------
def run_suite(args) -> None:
    """Times each hot-path kernel on the configuration it serves (SURVEY
    configs 1-5), with CUDA events around each launch, and reports achieved
    GB/s of algorithmic bytes against the measured HBM peak.

    Before every rep a 256 MiB buffer is written and then read: the write
    evicts the inputs from L2 (so the L2-resident config 1 starts cold), the
    read makes the flush's dirty lines drain to HBM before the timed launch
    instead of inside it.  `--only TEXT` keeps the entries whose
    "config: kernel" name contains TEXT (for profiler captures), `--warmup`
    sets the untimed reps before the timed ones."""
    import torch

    from tensorrs_b200 import abi, device

    torch.cuda.set_device(0)
    lib = abi.load()
    peak, peak_kind = measured_peaks()
    sh = torch.cuda.current_stream().cuda_stream
    flush_buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    f32 = torch.float32
    only = args.only
    warm = max(0, args.warmup)

    def want(cfg, name):
        return only is None or only in f"{cfg}: {name}"

    def t(*shape):
        return torch.empty(shape, dtype=f32, device="cuda")

    def timed(fn, reps):
        times = []
        for i in range(reps + warm):
            flush_buf.fill_(float(i))
            flush_buf.sum()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            if i >= warm:
                times.append(e0.elapsed_time(e1))
        return float(np.median(times))

    def run(cfg, name, nbytes, fn):
        if not want(cfg, name):
            return
        ms = timed(fn, reps)
        gbps = nbytes / (ms * 1e-3) / 1e9
        line = {"suite": cfg, "kernel": name, "bytes": int(nbytes), "ms": round(ms, 4), "GBps": round(gbps, 1),
                "frac_of_peak": round(gbps / peak, 4), "peak": peak, "peak_source": peak_kind,
                "l2": "256 MiB written then read before each rep"}
        print(json.dumps(line), flush=True)

    def any_of(cfg, names):
        return any(want(cfg, n) for n in names)

    def C(st):
        abi.check(st)

    V = device.view_of
    reps = max(5, args.steps)
    # config 1: A[1024,1024] + b[1024]; sum_axis(1); sum()
    c1 = ["bias add A[1024,1024] + b[1024]", "sum_axis(1) of A[1024,1024]", "sum() of A[1024,1024]"]
    if any_of("config1", c1):
        A = device.fill_uniform(t(1024, 1024), 0)
        b = device.fill_uniform(t(1024), 0, first=1 << 20)
        Y = t(1024, 1024)
        r = t(1024)
        s = t(1)
        va, vb, vy, vr, vs = V(A), V(b), V(Y), V(r), V(s)
        p2 = abi.program(2, abi.ADD)
        ins = abi.views_array([va, vb])
        run("config1", c1[0], 8392704, lambda: C(lib.trs_elementwise(ctypes.byref(p2), ins, ctypes.byref(vy), sh)))
        run("config1", c1[1], 4194304 + 4096, lambda: C(lib.trs_sum_axis(ctypes.byref(va), 1, 0, ctypes.byref(vr), sh)))
        run("config1", c1[2], 4194304 + 4, lambda: C(lib.trs_sum(ctypes.byref(va), ctypes.byref(vs), sh)))
        del A, b, Y
    # config 2: C = A & B^T, sigmoid
    c2 = ["A & B^T (B^T strided view)", "sigmoid(A & B^T) fused", "sigmoid standalone [4096,4096]"]
    if any_of("config2", c2):
        n = 4096
        A = device.fill_normal(t(n, n), 1)
        B = device.fill_normal(t(n, n), 1, first=n * n)
        Y = t(n, n)
        vbt = V(B, [n, n], [1, n], 0)
        nb = n * n * 4
        pm = abi.program(2, abi.MUL)
        pms = abi.program(2, abi.MUL, epilogue="sigmoid")
        ins = abi.views_array([V(A), vbt])
        vy = V(Y)
        run("config2", c2[0], 3 * nb, lambda: C(lib.trs_elementwise(ctypes.byref(pm), ins, ctypes.byref(vy), sh)))
        run("config2", c2[1], 3 * nb, lambda: C(lib.trs_elementwise(ctypes.byref(pms), ins, ctypes.byref(vy), sh)))
        params = (abi.Scalar * 2)()
        va = V(A)
        run("config2", c2[2], 2 * nb,
            lambda: C(lib.trs_unary(abi.UNOPS["sigmoid"], ctypes.byref(va), params, ctypes.byref(vy), sh)))
        del A, B, Y
    # config 3: X[8192,16384] axis reductions and softmax
    R, Cc = 8192, 16384
    c3 = [k for axis in (1, 0) for k in (f"sum_axis({axis}) of X[8192,16384]", f"mean over axis {axis}",
                                         f"max_axis({axis})", f"argmax_axis({axis})")] + ["softmax over axis 1"]
    if any_of("config3", c3):
        X = device.fill_normal(t(R, Cc), 2)
        vx = V(X)
        xb = R * Cc * 4
        r1, r0 = t(R), t(Cc)
        i1, i0 = torch.empty(R, dtype=torch.int64, device="cuda"), torch.empty(Cc, dtype=torch.int64, device="cuda")
        for axis, out_f, out_i, nout in [(1, r1, i1, R), (0, r0, i0, Cc)]:
            vo, vi = V(out_f), V(out_i)
            run("config3", f"sum_axis({axis}) of X[8192,16384]", xb + 4 * nout,
                lambda: C(lib.trs_sum_axis(ctypes.byref(vx), axis, 0, ctypes.byref(vo), sh)))
            run("config3", f"mean over axis {axis}", xb + 4 * nout,
                lambda: C(lib.trs_mean_axis(ctypes.byref(vx), axis, 0, ctypes.byref(vo), sh)))
            run("config3", f"max_axis({axis})", xb + 4 * nout,
                lambda: C(lib.trs_max_axis(ctypes.byref(vx), axis, ctypes.byref(vo), sh)))
            run("config3", f"argmax_axis({axis})", xb + 8 * nout,
                lambda: C(lib.trs_argmax_axis(ctypes.byref(vx), axis, ctypes.byref(vi), sh)))
        Ys = t(R, Cc)
        vys = V(Ys)
        run("config3", "softmax over axis 1", 2 * xb,
            lambda: C(lib.trs_softmax_lastdim(ctypes.byref(vx), ctypes.byref(vys), sh)))
        del X, Ys
    # config 4: relu(X & s + b) forward; scale/bias gradients backward
    c4 = ["relu(X & s + b) fused forward", "scale+bias grads of relu(X & s + b), fused",
          "reduce_broadcast_grad g -> [1,256,1,1]"]
    if any_of("config4", c4):
        N, Ch, H, W = 64, 256, 56, 56
        X = device.fill_normal(t(N, Ch, H, W), 3)
        G = device.fill_normal(t(N, Ch, H, W), 3, first=N * Ch * H * W)
        sc = device.fill_uniform(t(1, Ch, 1, 1), 3, 0.5, 1.5)
        bi = device.fill_uniform(t(1, Ch, 1, 1), 3, -0.1, 0.1, first=Ch)
        Y = t(N, Ch, H, W)
        gs, gb = t(1, Ch, 1, 1), t(1, Ch, 1, 1)
        xb = N * Ch * H * W * 4
        pf = abi.program(3, abi.MUL, abi.ADD, "relu")
        ins = abi.views_array([V(X), V(sc), V(bi)])
        vX, vG, vsc, vbi, vY, vgs, vgb = V(X), V(G), V(sc), V(bi), V(Y), V(gs), V(gb)
        run("config4", c4[0], 2 * xb + 2 * 4 * Ch,
            lambda: C(lib.trs_elementwise(ctypes.byref(pf), ins, ctypes.byref(vY), sh)))
        run("config4", c4[1], 2 * xb + 4 * 4 * Ch,
            lambda: C(lib.trs_affine_relu_backward(ctypes.byref(vG), ctypes.byref(vX), ctypes.byref(vsc),
                                                   ctypes.byref(vbi), ctypes.byref(vgs), ctypes.byref(vgb), sh)))
        tgt = (ctypes.c_int64 * 4)(1, Ch, 1, 1)
        run("config4", c4[2], xb + 4 * Ch,
            lambda: C(lib.trs_reduce_broadcast_grad(ctypes.byref(vG), tgt, 4, ctypes.byref(vgb), sh)))
        del X, G, Y
    # callers of the path: the pooling layers over config 4's activation
    cp = ["max_pool2d 2x2 over X[64,256,56,56]", "avg_pool2d 2x2 over X[64,256,56,56]",
          "max_pool2d 3x3 stride 2 over X[64,256,56,56]", "max_pool2d 2x2 backward to X[64,256,56,56]"]
    if any_of("callers", cp):
        N, Ch, H, W = 64, 256, 56, 56
        X = device.fill_normal(t(N, Ch, H, W), 3)
        P2, P3, GX = t(N, Ch, 28, 28), t(N, Ch, 27, 27), t(N, Ch, H, W)
        G2 = device.fill_normal(t(N, Ch, 28, 28), 11)
        xb, ob2, ob3 = N * Ch * H * W * 4, N * Ch * 28 * 28 * 4, N * Ch * 27 * 27 * 4
        vX, vP2, vP3, vG2, vGX = V(X), V(P2), V(P3), V(G2), V(GX)
        run("callers", cp[0], xb + ob2, lambda: C(lib.trs_max_pool2d(ctypes.byref(vX), 2, 2, 2, 2, ctypes.byref(vP2), sh)))
        run("callers", cp[1], xb + ob2, lambda: C(lib.trs_avg_pool2d(ctypes.byref(vX), 2, 2, 2, 2, ctypes.byref(vP2), sh)))
        run("callers", cp[2], xb + ob3, lambda: C(lib.trs_max_pool2d(ctypes.byref(vX), 3, 3, 2, 2, ctypes.byref(vP3), sh)))
        run("callers", cp[3], 2 * xb + ob2,
            lambda: C(lib.trs_max_pool2d_backward(ctypes.byref(vX), ctypes.byref(vG2), 2, 2, 2, 2, 0,
                                                  ctypes.byref(vGX), sh)))
        del X, P2, P3, GX, G2
    # callers of the path: LayerNorm over config 3's X, one Adam step over 2^26 f32 parameters
    cc = ["layer_norm over X[8192,16384]", "adam step, 2^26 f32 params", "sgd step, 2^26 f32 params"]
    if any_of("callers", cc):
        R, Cc = 8192, 16384
        X = device.fill_normal(t(R, Cc), 2)
        Yl = t(R, Cc)
        gam = device.fill_uniform(t(1, Cc), 7, 0.5, 1.5)
        bet = device.fill_uniform(t(1, Cc), 8, -0.5, 0.5)
        vX, vY, vg, vb = V(X), V(Yl), V(gam), V(bet)
        run("callers", cc[0], 2 * R * Cc * 4 + 2 * Cc * 4,
            lambda: C(lib.trs_layer_norm_lastdim(ctypes.byref(vX), ctypes.byref(vg), ctypes.byref(vb), 1e-5,
                                                 ctypes.byref(vY), sh)))
        del X, Yl
        n = 1 << 26
        P = device.fill_normal(t(n), 9)
        G = device.fill_normal(t(n), 10)
        M = torch.zeros(n, dtype=f32, device="cuda")
        W = torch.zeros(n, dtype=f32, device="cuda")
        vP, vG, vM, vW = V(P), V(G), V(M), V(W)
        step = [0]

        def adam():
            step[0] += 1
            C(lib.trs_adam_step(ctypes.byref(vP), ctypes.byref(vG), ctypes.byref(vM), ctypes.byref(vW), 1e-3, 0.9,
                                0.999, 1e-8, step[0], sh))
        run("callers", cc[1], 7 * n * 4, adam)
        run("callers", cc[2], 3 * n * 4, lambda: C(lib.trs_sgd_step(ctypes.byref(vP), ctypes.byref(vG), 1e-3, sh)))
        del P, G, M, W
    # config 5 (one GPU): the headline step
    c5 = ["Y = A & B + c and sum(Y) fused", "sum(Y) alone [65536,32768]"]
    if any_of("config5", c5):
        rows = args.rows
        A = device.fill_uniform(t(rows, COLS), SEED_A)
        B = device.fill_uniform(t(rows, COLS), SEED_B)
        c = device.fill_uniform(t(COLS), SEED_C)
        Y = t(rows, COLS)
        s = t(1)
        p3 = abi.program(3, abi.MUL, abi.ADD)
        ins = abi.views_array([V(A), V(B), V(c)])
        vY, vs = V(Y), V(s)
        run("config5", c5[0], workload_bytes(rows, COLS, 1),
            lambda: C(lib.trs_elementwise_sum(ctypes.byref(p3), ins, ctypes.byref(vY), ctypes.byref(vs), sh)))
        run("config5", c5[1], rows * COLS * 4 + 4, lambda: C(lib.trs_sum(ctypes.byref(vY), ctypes.byref(vs), sh)))


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.suite:
        run_suite(args)
    else:
        run_trs(args)


if __name__ == "__main__":
    main()
