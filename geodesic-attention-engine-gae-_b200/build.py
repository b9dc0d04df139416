"""Builds libgae.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python geodesic-attention-engine-gae-_b200/build.py [--force]

One translation unit (csrc/gae_abi.cu includes the kernel headers), static
CUDA runtime, no dependency on torch.  The output lands in lib/ next to this
file so that it travels with the source tree.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgae.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-diag-suppress", "177",
]


def _sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) +
                  glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


TRACE_LIB_PATH = os.path.join(LIB_DIR, "libgae_trace.so")


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    """Builds lib/libgae.so, or with trace=True the diagnostics variant
    lib/libgae_trace.so whose attention kernel records pipeline cycle stamps
    (include/gae_debug.h)."""
    out = TRACE_LIB_PATH if trace else LIB_PATH
    if not force and not trace and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = out + ".tmp"
    cmd = [NVCC, *NVCC_FLAGS, *(["-DGAE_ATTN_TRACE"] if trace else []),
           os.path.join(HERE, "csrc", "gae_abi.cu"), "-o", tmp]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, trace="--trace" in sys.argv))
