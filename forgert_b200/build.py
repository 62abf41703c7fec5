"""Builds libforgert_b200.so (the CUDA kernels + C ABI) in-tree for sm_100a.

Usage: python -m forgert_b200.build [--verbose]
The library is written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libforgert_b200.so"
SOURCES = [CSRC / "capi.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted((PKG_DIR.parent / "include").glob("*.h"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libforgert_b200.so")


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


# The trace variant (per-CTA phase timestamps, forgert_b200/phase_trace.py):
# the same sources with -DFR_TRACE, never loaded unless FORGERT_B200_LIB
# names it.
TRACE_LIB_PATH = PKG_DIR / "libforgert_b200_trace.so"


def build(verbose: bool = False, force: bool = False, trace: bool = False) -> Path:
    out = TRACE_LIB_PATH if trace else LIB_PATH
    if not force and not trace and not needs_build():
        return LIB_PATH
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS]
    if trace:
        cmd += ["-DFR_TRACE"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in SOURCES] + ["-o", str(tmp), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True, trace="--trace" in sys.argv))
