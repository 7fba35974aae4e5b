"""Builds libtrs_b200.so (the C ABI of include/trs.h) in-tree for sm_100a.

    python -m tensorrs_b200.build          # incremental
    python -m tensorrs_b200.build --clean  # from scratch

CUDA sources are compiled by nvcc for `-gencode arch=compute_100a,code=sm_100a`
with IEEE-exact arithmetic (no FMA contraction, no flush-to-zero, IEEE
division and square root); host sources by the system g++.  Objects go to
tensorrs_b200/_build/, the library to tensorrs_b200/libtrs_b200.so.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtrs_b200.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off",
             "-Wall", "-Wno-unused-function"]


def _cxx() -> str:
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def _compile(src: Path, verbose: bool, build_dir: Path = BUILD, defines: tuple = ()) -> Path:
    obj = build_dir / (src.name + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    inc = ["-I", str(CSRC), "-I", str(ROOT / "include"), "-I", str(CUDA_HOME / "include")]
    inc += [f"-D{d}" for d in defines]
    if src.suffix == ".cu":
        cmd = [str(CUDA_HOME / "bin" / "nvcc"), *ARCH, *NVCC_FLAGS, *inc, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [_cxx(), *CXX_FLAGS, *inc, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(clean: bool = False, verbose: bool = False, build_dir: Path = BUILD, lib: Path = LIB,
          defines: tuple = ()) -> Path:
    """Compiles every source into build_dir and links `lib`.  `defines` are
    extra -D macros (tuning knobs of the kernels; the defaults are the
    shipped configuration)."""
    if clean and build_dir.exists():
        shutil.rmtree(build_dir)
    build_dir.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, build_dir, defines), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not lib.exists() or lib.stat().st_mtime < newest:
        cmd = [str(CUDA_HOME / "bin" / "nvcc"), *ARCH, "-shared", "-o", str(lib), *map(str, objs),
               "-cudart", "static", "-ldl", "-lpthread", "-lrt",
               "-Xlinker", "--version-script=" + str(CSRC / "exports.map")]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"linking {lib.name} failed:\n{r.stdout}\n{r.stderr}")
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose=a.verbose))


if __name__ == "__main__":
    main()
