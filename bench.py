"""Benchmark of the broadcast-elementwise / full-reduction hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl trs|reference]
    python bench.py --suite      # every kernel of the path on its configuration

Default workload (the sharded configuration, run at 1/2/4/8 GPUs):
    Y = A & B + c, s = sum(Y)  with A, B f32 [65536, 32768] ~ U(-1,1) (8 GiB
    each), c f32 [32768] ~ U(-1,1), seed 4; A and B split on dim 0 across the
    ranks (strong scaling: the total problem is fixed), the ranks' f64
    partial sums combined over NVLink peer memory by the kernel that folds
    them (ncclAllReduce where peer mapping is unavailable).
A step is one fused pass through the C ABI (trs_elementwise_sum, or
trs_sharded_elementwise_sum for N > 1): Y written, sum(Y) returned.

The metric is achieved HBM bandwidth: algorithmic bytes (every tensor read
once at its stored size, every output written once) / time, whole job.
`value` times device-resident inputs with CUDA events (max over ranks);
`e2e` times the same call with host buffers, the host->device copies of A, B
and c and the device->host read of the sum inside the timed region.  Inputs
(8 GiB per operand) exceed the 126 MB L2, so no flush is needed.

At N = 1 the line also carries `suite`: every other kernel of the path timed
on its own configuration (see run_suite_entries).

--impl reference times the reference's own CPU algorithm (its restatement in
oracle/, with all host threads) on one dim-0 shard of the same workload.
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
    ap.add_argument("--no-steady", action="store_true",
                    help="with --suite: one flushed launch per kernel only (for profiler captures)")
    ap.add_argument("--no-suite", action="store_true",
                    help="leave the per-kernel suite out of the headline line")
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
    + c, packed_data + serial fold for sum) on one dim-0 shard of the
    workload, [8192, 32768]: 1/8 of the rows, which the full configuration's
    index vectors (about 72 GiB) need not fit in host memory.  At least two
    passes, and as many as fit in `seconds`; the full workload's time is 8x a
    pass, its GB/s the same."""
    import oracle
    oracle.set_threads(threads)
    rows = ROWS // 8
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
        del t
        oracle.sum_all(oracle.HostView(y.reshape(-1), [rows, COLS]))
        del y
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 2:
            break
    sec = float(np.median(times))
    nbytes = workload_bytes(rows, COLS, 1)
    return {
        "value": round(nbytes / sec / 1e9, 3), "unit": "GB/s", "cores": threads,
        "kind": "port",
        "sample": f"one dim-0 shard, {rows} of {ROWS} rows ([{rows},{COLS}] f32, 1/8 of the workload), "
                  f"{len(times)} timed passes, median {sec * 1e3:.0f} ms/pass (the full workload: 8x that); "
                  f"C++ restatement of binary_op/storage_indices/sum (oracle/oracle.cpp) on {threads} "
                  f"OpenMP threads",
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
                   "timed": "one [8192,32768] dim-0 shard per pass on the host cores"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region.

    An NVML thread in this process (the GPU matched to the CUDA device by its
    UUID) reads the SM clock, its maximum and the active clock-event reasons
    every 2 ms while `active` is set -- from just before the first timed
    launch to the synchronisation after the last -- so a timed region of a
    few tens of milliseconds still gets samples and idle time around it gets
    none.  Without NVML it falls back to `nvidia-smi -lms 100` over the whole
    window."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.thread = None
        self.rows = []
        self.active = False

    def _nvml_handle(self, nv):
        import torch
        try:
            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            return nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._nvml_handle(nv)
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.done = threading.Event()
            probe = (nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM),
                     reasons(h))
            del probe  # the calls work on this GPU

            def sample():
                try:
                    self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                      nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), int(reasons(h))))
                except Exception:
                    pass

            def run():
                while not self.done.is_set():
                    if self.active:
                        sample()
                    self.done.wait(0.002)
            self.sample_now = sample

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        self.active = False
        if self.thread is not None:
            self.done.set()
            self.thread.join(timeout=5)
            source = "nvml, 2 ms, timed region only"
            if not self.rows:
                # a region shorter than the sampling interval: one sample just after it
                self.sample_now()
                source = "nvml, one sample at the end of a region shorter than 2 ms"
            if not self.rows:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": "nvml"}
            names = sorted({n for _, _, r in self.rows for n, bit in self.REASONS if r & bit})
            return {"sm_mhz": float(np.median([r[0] for r in self.rows])),
                    "sm_max_mhz": float(max(r[1] for r in self.rows)), "reasons": names,
                    "samples": len(self.rows), "source": source}
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
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, 100 ms"}


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
    exchange = world > 1 and communicator.peer_exchange

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
    launches0 = lib.trs_launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks.active = True
    t_start.record(stream)
    for i in range(args.steps):
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    t_end.record(stream)
    barrier()
    clocks.active = False
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

    # where a sharded step goes: each rank's own element-wise + sum pass with
    # no cross-rank combine, timed the same way; the sharded step above minus
    # the slowest rank's local pass is the combine plus the wait for the
    # slowest rank
    breakdown = None
    if world > 1:
        def local_step():
            abi.check(lib.trs_elementwise_sum(ctypes.byref(prog), ins, ctypes.byref(yv), ctypes.byref(sv), sh))
        for _ in range(2):
            local_step()
        barrier()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for _ in range(args.steps):
            local_step()
        l1.record(stream)
        barrier()
        mine_ms = torch.tensor([l0.elapsed_time(l1) / args.steps], dtype=torch.float64, device="cuda")
        every = [torch.zeros_like(mine_ms) for _ in range(world)]
        dist.all_gather(every, mine_ms)
        local = [round(float(t[0]), 4) for t in every]
        breakdown = {"local_pass_ms_per_rank": local, "sharded_step_ms": round(ms_step, 4),
                     "combine_and_skew_ms": round(ms_step - max(local), 4),
                     "skew_ms": round(max(local) - min(local), 4)}

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

    suite = None
    if rank == 0 and world == 1 and not args.no_suite:
        del A, B, Y
        torch.cuda.empty_cache()
        suite, _, _ = run_suite_entries(args)

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
                       "parallelism": f"dim-0 shards x{world}" + (
                           (", f64 partials combined over NVLink peer memory inside the fold kernel"
                            if exchange else ", f64 partials combined by ncclAllReduce") if world > 1 else "")},
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
            "step_breakdown": breakdown,
            "suite": suite,
            "suite_about": "every other kernel of the path on its configuration (configs 1-4 and the callers), "
                           "one GPU: us_flushed = one launch after an L2 flush; us_steady = back-to-back "
                           "launches over rotating buffer sets >= 4x L2, so each pays its outputs' write-back; "
                           "frac = steady algorithmic GB/s / peak; dram_ratio = ncu DRAM bytes / algorithmic "
                           "bytes of one cold launch (profiles/traffic.json)" if suite else None,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        communicator.destroy()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# the kernel suite: every kernel of the path on the configuration it serves
# ---------------------------------------------------------------------------
L2_BYTES = 126 * 1024 * 1024
ROTATE_BYTES = 4 * L2_BYTES  # the buffer sets one steady-state run cycles through


class SuiteGroup:
    """Kernels that share one set of input and output buffers.  `make()`
    allocates and fills one set (a dict of tensors); each entry is
    (name, algorithmic bytes, launch(set))."""

    def __init__(self, cfg, make, entries):
        self.cfg, self.make, self.entries = cfg, make, entries


def suite_groups(lib, abi, device, torch):
    """The hot-path kernels on their benchmark configurations (inputs drawn
    from the same seeded streams the parity tests use)."""
    f32 = torch.float32
    sh = torch.cuda.current_stream().cuda_stream
    V = device.view_of

    def t(*shape, dtype=f32):
        return torch.empty(shape, dtype=dtype, device="cuda")

    def C(st):
        abi.check(st)

    def ref(x):
        return ctypes.byref(x)

    groups = []

    # config 1: A[1024,1024] + b[1024]; sum_axis(1); sum()
    def make1():
        A = device.fill_uniform(t(1024, 1024), 0)
        b = device.fill_uniform(t(1024), 0, first=1 << 20)
        s = {"A": A, "b": b, "Y": t(1024, 1024), "r": t(1024), "s": t(1)}
        s["v"] = {k: V(x) for k, x in s.items() if isinstance(x, torch.Tensor)}
        s["ins"] = abi.views_array([s["v"]["A"], s["v"]["b"]])
        s["p"] = abi.program(2, abi.ADD)
        return s
    groups.append(SuiteGroup("config1", make1, [
        ("bias add A[1024,1024] + b[1024]", 8392704,
         lambda s: C(lib.trs_elementwise(ref(s["p"]), s["ins"], ref(s["v"]["Y"]), sh))),
        ("sum_axis(1) of A[1024,1024]", 4194304 + 4096,
         lambda s: C(lib.trs_sum_axis(ref(s["v"]["A"]), 1, 0, ref(s["v"]["r"]), sh))),
        ("sum() of A[1024,1024]", 4194304 + 4,
         lambda s: C(lib.trs_sum(ref(s["v"]["A"]), ref(s["v"]["s"]), sh))),
        # the chain the configuration names: y = A + b, y.sum_axis(1), y.sum()
        ("chain y = A + b, y.sum_axis(1), y.sum() as three calls", 8392704 + 4194304 + 4096 + 4194304 + 4,
         lambda s: (C(lib.trs_elementwise(ref(s["p"]), s["ins"], ref(s["v"]["Y"]), sh)),
                    C(lib.trs_sum_axis(ref(s["v"]["Y"]), 1, 0, ref(s["v"]["r"]), sh)),
                    C(lib.trs_sum(ref(s["v"]["Y"]), ref(s["v"]["s"]), sh)))),
        ("chain y = A + b, y.sum_axis(1), y.sum() in one pass", 8392704 + 4096 + 4,
         lambda s: C(lib.trs_elementwise_row_sums(ref(s["p"]), s["ins"], ref(s["v"]["Y"]), ref(s["v"]["r"]),
                                                  ref(s["v"]["s"]), sh))),
    ]))

    # config 2: C = A & B^T (B^T a strided view), sigmoid
    n = 4096
    nb = n * n * 4

    def make2():
        A = device.fill_normal(t(n, n), 1)
        B = device.fill_normal(t(n, n), 1, first=n * n)
        s = {"A": A, "B": B, "Y": t(n, n)}
        s["va"], s["vy"] = V(A), V(s["Y"])
        s["ins"] = abi.views_array([s["va"], V(B, [n, n], [1, n], 0)])
        s["pm"] = abi.program(2, abi.MUL)
        s["pms"] = abi.program(2, abi.MUL, epilogue="sigmoid")
        s["par"] = (abi.Scalar * 2)()
        return s
    groups.append(SuiteGroup("config2", make2, [
        ("A & B^T (B^T strided view)", 3 * nb,
         lambda s: C(lib.trs_elementwise(ref(s["pm"]), s["ins"], ref(s["vy"]), sh))),
        ("sigmoid(A & B^T) fused", 3 * nb,
         lambda s: C(lib.trs_elementwise(ref(s["pms"]), s["ins"], ref(s["vy"]), sh))),
        ("sigmoid standalone [4096,4096]", 2 * nb,
         lambda s: C(lib.trs_unary(abi.UNOPS["sigmoid"], ref(s["va"]), s["par"], ref(s["vy"]), sh))),
    ]))

    # config 3: X[8192,16384] axis reductions and softmax
    R, Cc = 8192, 16384
    xb = R * Cc * 4

    def make3():
        X = device.fill_normal(t(R, Cc), 2)
        s = {"X": X, "r1": t(R), "r0": t(Cc), "i1": t(R, dtype=torch.int64), "i0": t(Cc, dtype=torch.int64),
             "Y": t(R, Cc)}
        s["v"] = {k: V(x) for k, x in s.items()}
        return s
    e3 = []
    for axis, nout, of, oi in [(1, R, "r1", "i1"), (0, Cc, "r0", "i0")]:
        e3 += [
            (f"sum_axis({axis}) of X[8192,16384]", xb + 4 * nout,
             lambda s, a=axis, o=of: C(lib.trs_sum_axis(ref(s["v"]["X"]), a, 0, ref(s["v"][o]), sh))),
            (f"mean over axis {axis}", xb + 4 * nout,
             lambda s, a=axis, o=of: C(lib.trs_mean_axis(ref(s["v"]["X"]), a, 0, ref(s["v"][o]), sh))),
            (f"max_axis({axis})", xb + 4 * nout,
             lambda s, a=axis, o=of: C(lib.trs_max_axis(ref(s["v"]["X"]), a, ref(s["v"][o]), sh))),
            (f"argmax_axis({axis})", xb + 8 * nout,
             lambda s, a=axis, o=oi: C(lib.trs_argmax_axis(ref(s["v"]["X"]), a, ref(s["v"][o]), sh))),
        ]
    e3.append(("softmax over axis 1", 2 * xb,
               lambda s: C(lib.trs_softmax_lastdim(ref(s["v"]["X"]), ref(s["v"]["Y"]), sh))))
    groups.append(SuiteGroup("config3", make3, e3))

    # config 4: relu(X & s + b) forward; scale/bias gradients backward
    N, Ch, H, W = 64, 256, 56, 56
    x4 = N * Ch * H * W * 4

    def make4():
        X = device.fill_normal(t(N, Ch, H, W), 3)
        G = device.fill_normal(t(N, Ch, H, W), 3, first=N * Ch * H * W)
        sc = device.fill_uniform(t(1, Ch, 1, 1), 3, 0.5, 1.5)
        bi = device.fill_uniform(t(1, Ch, 1, 1), 3, -0.1, 0.1, first=Ch)
        s = {"X": X, "G": G, "sc": sc, "bi": bi, "Y": t(N, Ch, H, W), "gs": t(1, Ch, 1, 1), "gb": t(1, Ch, 1, 1)}
        s["v"] = {k: V(x) for k, x in s.items()}
        s["ins"] = abi.views_array([s["v"]["X"], s["v"]["sc"], s["v"]["bi"]])
        s["pf"] = abi.program(3, abi.MUL, abi.ADD, "relu")
        s["tgt"] = (ctypes.c_int64 * 4)(1, Ch, 1, 1)
        return s
    groups.append(SuiteGroup("config4", make4, [
        ("relu(X & s + b) fused forward", 2 * x4 + 2 * 4 * Ch,
         lambda s: C(lib.trs_elementwise(ref(s["pf"]), s["ins"], ref(s["v"]["Y"]), sh))),
        ("scale+bias grads of relu(X & s + b), fused", 2 * x4 + 4 * 4 * Ch,
         lambda s: C(lib.trs_affine_relu_backward(ref(s["v"]["G"]), ref(s["v"]["X"]), ref(s["v"]["sc"]),
                                                  ref(s["v"]["bi"]), ref(s["v"]["gs"]), ref(s["v"]["gb"]), sh))),
        ("reduce_broadcast_grad g -> [1,256,1,1]", x4 + 4 * Ch,
         lambda s: C(lib.trs_reduce_broadcast_grad(ref(s["v"]["G"]), s["tgt"], 4, ref(s["v"]["gb"]), sh))),
    ]))

    # callers of the path: pooling over config 4's activation
    o2, o3 = N * Ch * 28 * 28 * 4, N * Ch * 27 * 27 * 4

    def make_pool():
        X = device.fill_normal(t(N, Ch, H, W), 3)
        s = {"X": X, "P2": t(N, Ch, 28, 28), "P3": t(N, Ch, 27, 27), "GX": t(N, Ch, H, W),
             "G2": device.fill_normal(t(N, Ch, 28, 28), 11)}
        s["v"] = {k: V(x) for k, x in s.items()}
        return s
    groups.append(SuiteGroup("callers", make_pool, [
        ("max_pool2d 2x2 over X[64,256,56,56]", x4 + o2,
         lambda s: C(lib.trs_max_pool2d(ref(s["v"]["X"]), 2, 2, 2, 2, ref(s["v"]["P2"]), sh))),
        ("avg_pool2d 2x2 over X[64,256,56,56]", x4 + o2,
         lambda s: C(lib.trs_avg_pool2d(ref(s["v"]["X"]), 2, 2, 2, 2, ref(s["v"]["P2"]), sh))),
        ("max_pool2d 3x3 stride 2 over X[64,256,56,56]", x4 + o3,
         lambda s: C(lib.trs_max_pool2d(ref(s["v"]["X"]), 3, 3, 2, 2, ref(s["v"]["P3"]), sh))),
        ("max_pool2d 2x2 backward to X[64,256,56,56]", 2 * x4 + o2,
         lambda s: C(lib.trs_max_pool2d_backward(ref(s["v"]["X"]), ref(s["v"]["G2"]), 2, 2, 2, 2, 0,
                                                 ref(s["v"]["GX"]), sh))),
    ]))

    # callers of the path: LayerNorm over config 3's X; optimiser steps
    def make_ln():
        X = device.fill_normal(t(R, Cc), 2)
        s = {"X": X, "Y": t(R, Cc), "g": device.fill_uniform(t(1, Cc), 7, 0.5, 1.5),
             "b": device.fill_uniform(t(1, Cc), 8, -0.5, 0.5)}
        s["v"] = {k: V(x) for k, x in s.items()}
        return s
    groups.append(SuiteGroup("callers", make_ln, [
        ("layer_norm over X[8192,16384]", 2 * R * Cc * 4 + 2 * Cc * 4,
         lambda s: C(lib.trs_layer_norm_lastdim(ref(s["v"]["X"]), ref(s["v"]["g"]), ref(s["v"]["b"]), 1e-5,
                                                ref(s["v"]["Y"]), sh))),
    ]))
    npar = 1 << 26

    def make_opt():
        s = {"P": device.fill_normal(t(npar), 9), "G": device.fill_normal(t(npar), 10),
             "M": torch.zeros(npar, dtype=f32, device="cuda"), "W": torch.zeros(npar, dtype=f32, device="cuda")}
        s["v"] = {k: V(x) for k, x in s.items()}
        s["step"] = [0]
        return s

    def adam(s):
        s["step"][0] += 1
        C(lib.trs_adam_step(ref(s["v"]["P"]), ref(s["v"]["G"]), ref(s["v"]["M"]), ref(s["v"]["W"]), 1e-3, 0.9,
                            0.999, 1e-8, s["step"][0], sh))
    groups.append(SuiteGroup("callers", make_opt, [
        ("adam step, 2^26 f32 params", 7 * npar * 4, adam),
        ("sgd step, 2^26 f32 params", 3 * npar * 4,
         lambda s: C(lib.trs_sgd_step(ref(s["v"]["P"]), ref(s["v"]["G"]), 1e-3, sh))),
    ]))

    # callers of the path: matmul (Linear, Conv2d) and the im2col pair
    mm = 4096

    def make_mm():
        s = {"A": device.fill_normal(t(mm, mm), 14), "B": device.fill_normal(t(mm, mm), 15), "C": t(mm, mm)}
        s["v"] = {k: V(x) for k, x in s.items()}
        return s
    groups.append(SuiteGroup("callers", make_mm, [
        ("matmul [4096,4096] x [4096,4096] f32, reference order", 3 * mm * mm * 4,
         lambda s: C(lib.trs_matmul(ref(s["v"]["A"]), ref(s["v"]["B"]), ref(s["v"]["C"]), sh)), 2 * mm ** 3),
        ("matmul_tf32x3 [4096,4096] x [4096,4096] f32, tensor cores", 3 * mm * mm * 4,
         lambda s: C(lib.trs_matmul_tf32x3(ref(s["v"]["A"]), ref(s["v"]["B"]), ref(s["v"]["C"]), sh)),
         2 * mm ** 3, "tc"),
    ]))
    cN, cC, cH, cW = 32, 64, 56, 56
    crow, cpatch = cN * cH * cW, cC * 9
    xb_c, cb_c = cN * cC * cH * cW * 4, crow * cpatch * 4

    def make_cols():
        s = {"X": device.fill_normal(t(cN, cC, cH, cW), 16), "K": t(crow, cpatch), "Y": t(cN, cC, cH, cW)}
        s["v"] = {k: V(x) for k, x in s.items()}
        return s
    groups.append(SuiteGroup("callers", make_cols, [
        ("unfold_2d 3x3 pad 1 of X[32,64,56,56]", xb_c + cb_c,
         lambda s: C(lib.trs_unfold_2d(ref(s["v"]["X"]), 3, 3, 1, 1, 1, 1, ref(s["v"]["K"]), sh))),
        ("fold_2d 3x3 pad 1 into X[32,64,56,56]", xb_c + cb_c,
         lambda s: C(lib.trs_fold_2d(ref(s["v"]["K"]), 3, 3, 1, 1, 1, 1, ref(s["v"]["Y"]), sh))),
    ]))
    return groups


def tf32_tensor_peak() -> float:
    """Dense TF32 tensor-core operations per second: half the measured bf16
    rate (MEASURED_PEAKS.json bf16_tflops; TF32 runs at half the bf16 rate)."""
    tf = 1679.4
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        tf = float(json.loads(p.read_text()).get("bf16_tflops", tf))
    except (OSError, ValueError):
        pass
    return tf * 1e12 / 2


def fp32_lane_peak() -> float:
    """FP32 lane operations per second of the CUDA cores at the measured
    maximum SM clock: 148 SMs x 128 lanes x clock.  matmul in the reference's
    order spends two of them per multiply-add (a separately rounded product
    and sum), so 2 M N K flops against this figure is its compute roofline."""
    mhz = 1965.0
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        mhz = float(json.loads(p.read_text()).get("sm_max_mhz", mhz))
    except (OSError, ValueError):
        pass
    return 148 * 128 * mhz * 1e6


def set_bytes(s) -> int:
    import torch
    return sum(x.numel() * x.element_size() for x in s.values() if isinstance(x, torch.Tensor))


def suite_traffic() -> dict:
    """DRAM bytes per launch of each suite kernel (read + write, one cold
    launch under ncu), from profiles/traffic.json."""
    p = ROOT / "profiles" / "traffic.json"
    try:
        return json.loads(p.read_text()).get("suite", {})
    except (OSError, ValueError):
        return {}


def run_suite_entries(args, only=None, steady=True, flushed_reps=5, warm=2):
    """Times every suite kernel two ways, with CUDA events on the launching
    stream, and returns one record per kernel:
      * flushed: one launch after a 256 MiB buffer was written and then read
        (the write evicts the inputs from L2, the read drains the flush's
        dirty lines to HBM before the timed launch rather than inside it) --
        a cold start, launch latency included, but the output may still sit
        in the 126 MB L2 when the kernel ends;
      * steady: launches back to back over rotating copies of the inputs and
        outputs totalling at least 4x L2 (504 MiB), timed as a whole and
        divided by the launch count -- each launch pays for the write-back of
        the outputs before it, so algorithmic bytes / this time is what HBM
        sustains.
    `frac` is steady algorithmic GB/s over the measured copy peak; `dram_ratio`
    is the kernel's DRAM traffic under ncu over its algorithmic bytes."""
    import torch

    from tensorrs_b200 import abi, device

    lib = abi.load()
    peak, peak_kind = measured_peaks()
    stream = torch.cuda.current_stream()
    flush_buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    traffic = suite_traffic()
    out = []

    def ev():
        return torch.cuda.Event(enable_timing=True)

    for g in suite_groups(lib, abi, device, torch):
        names = [e for e in g.entries if only is None or only in f"{g.cfg}: {e[0]}"]
        if not names:
            continue
        sets = [g.make()]
        sb = set_bytes(sets[0])
        if steady:
            n_sets = min(64, max(2, -(-ROTATE_BYTES // max(sb, 1))))
            sets += [g.make() for _ in range(n_sets - 1)]
        torch.cuda.synchronize()
        for entry in names:
            name, nbytes, launch = entry[:3]
            flops = entry[3] if len(entry) > 3 else None
            times = []
            for i in range(flushed_reps + warm):
                flush_buf.fill_(float(i))
                flush_buf.sum()
                e0, e1 = ev(), ev()
                e0.record(stream)
                launch(sets[0])
                e1.record(stream)
                e1.synchronize()
                if i >= warm:
                    times.append(e0.elapsed_time(e1))
            ms_f = float(np.median(times))
            rec = {"suite": g.cfg, "kernel": name, "bytes": int(nbytes), "us_flushed": round(ms_f * 1e3, 2),
                   "frac_flushed": round(nbytes / (ms_f * 1e-3) / 1e9 / peak, 4)}
            if steady:
                k = len(sets)
                n_launch = max(2 * k, 20)
                for i in range(k):
                    launch(sets[i])
                e0, e1 = ev(), ev()
                e0.record(stream)
                for i in range(n_launch):
                    launch(sets[i % k])
                e1.record(stream)
                e1.synchronize()
                ms_s = e0.elapsed_time(e1) / n_launch
                gbps = nbytes / (ms_s * 1e-3) / 1e9
                rec.update({"us_steady": round(ms_s * 1e3, 2), "GBps": round(gbps, 1), "frac": round(gbps / peak, 4),
                            "rotation": f"{k} buffer sets x {sb / 2**20:.0f} MiB"})
            if flops:  # a contraction: its roofline is compute, not HBM
                ms = rec.get("us_steady", rec["us_flushed"]) / 1e3
                tf = flops / (ms * 1e-3) / 1e12
                if len(entry) > 4 and entry[4] == "tc":
                    # three TF32 products per multiply-add (hi*hi, hi*lo, lo*hi)
                    peak_ops, hw = tf32_tensor_peak(), 3.0
                    bound = "tensor cores (tcgen05 kind::tf32, three products per multiply-add)"
                else:
                    peak_ops, hw = fp32_lane_peak(), 1.0
                    bound = "fp32 CUDA cores (separately rounded multiply and add)"
                rec.update({"flops": int(flops), "TFLOPs": round(tf, 2), "frac": round(hw * tf * 1e12 / peak_ops, 4),
                            "bound": bound})
                rec.pop("GBps", None)
                rec["frac_flushed"] = round(hw * flops / (ms_f * 1e-3) / peak_ops, 4)
            tr = traffic.get(name)
            rec["dram_ratio"] = round(tr / nbytes, 3) if tr else None
            out.append(rec)
        del sets
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out, peak, peak_kind


def run_suite(args) -> None:
    """--suite: one JSON line per kernel of the path (run_suite_entries), plus
    the headline configuration's fused step and its sum alone."""
    import torch

    from tensorrs_b200 import abi, device

    torch.cuda.set_device(0)
    recs, peak, peak_kind = run_suite_entries(
        args, only=args.only, steady=not args.no_steady,
        flushed_reps=max(1, args.steps) if args.no_steady else max(5, args.steps), warm=max(0, args.warmup))
    for r in recs:
        r.update({"peak": peak, "peak_source": peak_kind})
        print(json.dumps(r), flush=True)
    # the headline configuration (24 GiB on the device): only in timing runs,
    # never in a single-launch profiler pass
    c5 = ["Y = A & B + c and sum(Y) fused", "sum(Y) alone [65536,32768]"]
    if args.no_steady or (args.only is not None and not any(args.only in f"config5: {n}" for n in c5)):
        return
    lib = abi.load()
    sh = torch.cuda.current_stream().cuda_stream
    f32 = torch.float32
    rows = args.rows
    A = device.fill_uniform(torch.empty((rows, COLS), dtype=f32, device="cuda"), SEED_A)
    B = device.fill_uniform(torch.empty((rows, COLS), dtype=f32, device="cuda"), SEED_B)
    c = device.fill_uniform(torch.empty((COLS,), dtype=f32, device="cuda"), SEED_C)
    Y = torch.empty((rows, COLS), dtype=f32, device="cuda")
    s = torch.empty((1,), dtype=f32, device="cuda")
    p3 = abi.program(3, abi.MUL, abi.ADD)
    ins = abi.views_array([device.view_of(A), device.view_of(B), device.view_of(c)])
    vY, vs = device.view_of(Y), device.view_of(s)
    for name, nbytes, fn in [
            (c5[0], workload_bytes(rows, COLS, 1),
             lambda: abi.check(lib.trs_elementwise_sum(ctypes.byref(p3), ins, ctypes.byref(vY), ctypes.byref(vs), sh))),
            (c5[1], rows * COLS * 4 + 4, lambda: abi.check(lib.trs_sum(ctypes.byref(vY), ctypes.byref(vs), sh)))]:
        if args.only is not None and args.only not in f"config5: {name}":
            continue
        for _ in range(max(1, args.warmup)):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(5, args.steps)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        gbps = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"suite": "config5", "kernel": name, "bytes": int(nbytes), "us_steady": round(ms * 1e3, 1),
                          "GBps": round(gbps, 1), "frac": round(gbps / peak, 4), "peak": peak,
                          "peak_source": peak_kind, "l2": "inputs 8 GiB per operand >> L2"}), flush=True)


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
