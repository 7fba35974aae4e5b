"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run on a B200; the
rest run on CPU (oracle, host planning, library loading)."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_kats.json"
NP_DTYPES = {"f32": np.float32, "f64": np.float64, "i32": np.int32, "i64": np.int64}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


def golden_cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.load()
    return oracle


@pytest.fixture(scope="session")
def trs():
    from tensorrs_b200 import abi
    abi.load()
    return abi
