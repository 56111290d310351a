#!/usr/bin/env python3
"""Build libtk_b200.so in-tree for sm_100a.

    python transformer-kernel_b200/build.py [--force] [--verbose]

One translation unit (csrc/tk_abi.cu includes every kernel) compiled with
nvcc -gencode arch=compute_100a,code=sm_100a into
transformer-kernel_b200/libtk_b200.so, next to the Python modules that load
it with ctypes. The CUDA runtime is linked statically; the driver API is
reached through cudaGetDriverEntryPoint, so no -lcuda is needed. Rebuilds
only when a source under csrc/ or include/ is newer than the library.
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
LIB = HERE / "libtk_b200.so"
SOURCES = [HERE / "csrc" / "tk_abi.cu"]
DEPS = sorted((HERE / "csrc").glob("*.cu*")) + sorted((ROOT / "include").glob("*.h"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-Xptxas", "-v",
    "--expt-relaxed-constexpr",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not pathlib.Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, SOURCES)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
