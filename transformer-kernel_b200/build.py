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
import re
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


def kernel_resources(ptxas_log: str) -> dict:
    """{mangled kernel name: (registers, spill store bytes, stack frame bytes)}
    from ptxas -v output. Stack and spill figures are keyed by the function a
    "Function properties for X" line names (a non-inlined device function's
    block never counts against the kernel compiled before it); register
    counts by the entry function being compiled."""
    regs, frame, entry, props = {}, {}, None, None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            entry, props = m.group(1), None
            continue
        m = re.search(r"Function properties for (\S+)", line)
        if m:
            props = m.group(1)
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores", line)
        if m and props:
            frame[props] = (int(m.group(2)), int(m.group(1)))
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and entry:
            regs[entry] = int(m.group(1))
    return {name: (r, *frame.get(name, (0, 0))) for name, r in regs.items()}


def check_register_split(ptxas_log: str) -> None:
    """The persistent attention kernel splits its launch allocation with
    setmaxnreg (csrc/tk_attn.cuh kLaunchRegs): it must build with exactly
    that many registers per thread, without spills and without a stack frame
    (local memory would be reached through the reduced register budget)."""
    text = (HERE / "csrc" / "tk_attn.cuh").read_text()
    want = int(re.search(r"constexpr int kLaunchRegs = (\d+);", text).group(1))
    found = {k: v for k, v in kernel_resources(ptxas_log).items() if "attn15attn_fwd_kernel" in k}
    if not found:
        raise RuntimeError("ptxas output lists no attn_fwd_kernel")
    bad = {k: v for k, v in found.items() if v != (want, 0, 0)}
    if bad:
        raise RuntimeError(f"attn_fwd_kernel needs {want} registers, no spills and no stack frame for its register "
                           f"split; ptxas gave (registers, spill bytes, stack bytes) {sorted(bad.values())}")


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
    check_register_split(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
