"""Several GPUs: the trs_sharded_* entry points on 2 (or more) ranks, one
process per GPU over NCCL, against the oracle on the unsplit tensor (see
_sharded_worker.py for the cases and tolerances), and communicator creation
failing with TRS_ERR_TIMEOUT when a rank never joins.

These launch child processes: a failure ends a child with an error, never a
GPU kernel that waits on a rank that is gone (every collective here runs
between ranks that are all alive; the timeout case never gets as far as a
collective).  The one wait made to run out on purpose is the sharded sum's
peer exchange, where rank 1 skips a call while staying alive: rank 0's kernel
gives up after its bounded wait (about 2 s) and reports it in the async-error
word.  The exchange uses plain peer stores and loads (no multicast); NCCL's
NVLink SHARP path is switched off in the children."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child_env() -> dict:
    env = dict(os.environ)
    env["NCCL_NVLS_ENABLE"] = "0"
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT), str(ROOT / "tests"), env.get("PYTHONPATH", "")])
    return env


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_sharded_entry_points_on_two_ranks(tmp_path):
    world = 2
    cmd = ["timeout", "-k", "20", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "_sharded_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=_child_env(), capture_output=True, text=True, timeout=460)
    reports = {}
    for k in range(world):
        p = tmp_path / f"rank{k}.json"
        if p.exists():
            reports[k] = json.loads(p.read_text())
    assert r.returncode == 0 and len(reports) == world, (r.returncode, r.stdout[-3000:], r.stderr[-3000:], reports)
    for k, rep in reports.items():
        assert rep["failures"] == [], (k, rep["failures"][:5])
        # B200s under NVSwitch map each other's memory: the full sums combine
        # over NVLink peer memory, not through NCCL
        assert rep["peer_exchange"], k


TIMEOUT_CHILD = r"""
import ctypes, sys, time
from tensorrs_b200 import abi
lib = abi.load()
uid = (ctypes.c_uint8 * 128)()
abi.check(lib.trs_comm_unique_id(uid))
comm = ctypes.c_void_p()
t0 = time.monotonic()
st = lib.trs_comm_init_rank(uid, 2, 0, 3000, ctypes.byref(comm))
dt = time.monotonic() - t0
print(st, round(dt, 2), abi.last_error())
sys.exit(0 if st == abi.ERR_TIMEOUT and 2.5 <= dt <= 30 and not comm.value else 1)
"""


@pytest.mark.skipif(_gpus() < 1, reason="needs a GPU")
def test_comm_init_times_out_when_a_rank_never_joins():
    """Rank 1 of a 2-rank communicator never calls in: rank 0's creation
    returns TRS_ERR_TIMEOUT after its 3 s deadline and aborts the half-made
    communicator (host-side only: no collective is ever launched)."""
    r = subprocess.run([sys.executable, "-c", TIMEOUT_CHILD], env=_child_env(), capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
