"""Build libsm100_fp8_wgrad.so (sm_100a) in-tree with nvcc.

Usage: python sm90-fp8-wgrad_b200/build_ext.py [--force] [--profile]
Output: sm90-fp8-wgrad_b200/sm90_fp8_wgrad/_lib/libsm100_fp8_wgrad.so
        (--profile: libsm100_fp8_wgrad_profile.so with the GEMM's per-role cycle
        counters, -DWGRAD_PROFILE=1, read with sm90_fp8_wgrad._lib.profile_counters();
        --debug-modes: libsm100_fp8_wgrad_debug.so with the known-answer kernel
        modes of KERNEL_LAB_WGRAD_KERNEL_MODE, -DWGRAD_DEBUG_MODES=1. Load either
        with SM100_WGRAD_LIB=<path>.
        --trace N: libsm100_fp8_wgrad_trace.so with per-K-block clock64 event
        stamps of CTAs 0 and 1 (-DWGRAD_TRACE=N: 1 MMA issuer + promotion warp,
        2 per-chunk promotion stamps), printed by python -m sm90_fp8_wgrad.timeline.)
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad.so"
OUT_PROFILE = HERE / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad_profile.so"
OUT_DEBUG = HERE / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad_debug.so"
OUT_TRACE = HERE / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad_trace{}.so"
SOURCES = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "sm100_fp8_wgrad.h"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def needs_build(out: Path = OUT) -> bool:
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    return any(s.stat().st_mtime > mtime for s in SOURCES)


def build(force: bool = False, verbose: bool = False, profile: bool = False, debug_modes: bool = False,
          trace: int = 0) -> Path:
    out = Path(str(OUT_TRACE).format(trace)) if trace else (OUT_DEBUG if debug_modes else (OUT_PROFILE if profile else OUT))
    if not force and not needs_build(out):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-v" if verbose else "-O3",
        *(["-DWGRAD_PROFILE=1"] if profile else []),
        *(["-DWGRAD_DEBUG_MODES=1"] if debug_modes else []),
        *([f"-DWGRAD_TRACE={int(trace)}"] if trace else []),
        "-o", str(tmp), str(CSRC / "unity.cu"),
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--profile", action="store_true", help="build the per-role cycle-counter library")
    ap.add_argument("--debug-modes", action="store_true", help="build the known-answer kernel-mode library")
    ap.add_argument("--trace", type=int, choices=(1, 2), default=0, help="build the event-trace library")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, profile=a.profile, debug_modes=a.debug_modes, trace=a.trace))
