"""Build libsdtw_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m softdtw_cuda._build          (from sdtw-cuda-torch_b200/)

The library lands in softdtw_cuda/_lib/ next to this file, where
softdtw_cuda._native loads it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # sdtw-cuda-torch_b200/
CSRC = os.path.join(ROOT, "csrc")
LIB_DIR = os.path.join(PKG, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libsdtw_b200.so")

SOURCES = ["capi.cu", "wavefront.cu", "wavefront_exp.cu", "layout.cu", "dense.cu", "tcgemm.cu", "grad_small.cu", "barycenter.cu", "f64.cu", "cpu.cpp"]
HEADERS = ["sdtw_device.cuh", "sdtw_kernels.h", "sdtw_plan.h", "wavefront_ring.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsdtw_b200.so")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(os.path.dirname(ROOT), "include", "sdtw_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fopenmp",
           "-shared", "-o", tmp] + [os.path.join(CSRC, f) for f in SOURCES] + ["-lgomp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    env = dict(os.environ)
    # nvcc's host compiler must have OpenMP; prefer the system gcc.
    if os.path.exists("/usr/bin/g++"):
        cmd[1:1] = ["-ccbin", "/usr/bin/g++"]
    subprocess.run(cmd, check=True, env=env)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
