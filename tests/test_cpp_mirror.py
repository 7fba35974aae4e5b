"""The C++ mirror of the reference's Tensor API (include/trs_tensor.hpp):
compiles here; its restatement of the reference's own unit tests runs on the
GPU."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

from conftest import ROOT

SRC = ROOT / "tests" / "cpp" / "test_tensor.cpp"
BIN = ROOT / "tests" / "cpp" / "_build" / "test_tensor"
LIBDIR = ROOT / "tensorrs_b200"


def compile_mirror_tests() -> Path:
    BIN.parent.mkdir(exist_ok=True)
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-I", str(ROOT / "include"), str(SRC), "-o", str(BIN),
           "-L", str(LIBDIR), "-ltrs_b200", f"-Wl,-rpath,{LIBDIR}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return BIN


def test_mirror_compiles_against_the_abi():
    assert compile_mirror_tests().exists()


@pytest.mark.gpu
def test_reference_unit_tests_pass_on_the_gpu():
    binary = compile_mirror_tests()
    r = subprocess.run([str(binary)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    print(r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
