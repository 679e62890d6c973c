"""Build recipe of the CUDA library: nvcc, sm_100a, in-tree output.

``build_library()`` compiles every ``csrc/*.cu`` into
``unbox.ai_b200/lib/libunbox_b200.so`` (static CUDA runtime, no torch
dependency). Run ``python -m`` style through ``__graft_entry__.build()`` or
directly: ``python unbox.ai_b200/build.py``.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libunbox_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def build_library(verbose_ptxas: bool = False, extra=None) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
           "-o", LIB_PATH, *sources()]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    if extra:
        cmd[1:1] = list(extra)
    subprocess.check_call(cmd)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(verbose_ptxas="-v" in sys.argv))
