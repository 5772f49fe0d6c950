"""Build recipe for the B200 grouped-GEMM library (nvcc, sm_100a only).

Outputs, in-tree so they travel with the repository snapshot:
  lib/libgg_b200.so   C ABI of include/gg_b200.h (static CUDA runtime)
  lib/gg_bench        C++ shapes-CSV -> results-CSV benchmark (bench_main contract)

Usage: python build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-I" + INCLUDE, "-I" + CSRC]

TARGETS = {
    "libgg_b200.so": {
        "srcs": ["gg_capi.cu"],
        "deps": ["gg_capi.cu", "gg_kernel.cuh", "gg_ptx.cuh"],
        "flags": ["-Xcompiler", "-fPIC", "-shared"],
    },
    "gg_bench": {
        "srcs": ["gg_bench_main.cu", "gg_cublas_backends.cpp", "gg_capi.cu"],
        "deps": ["gg_bench_main.cu", "gg_cublas_backends.cpp", "gg_capi.cu", "gg_kernel.cuh", "gg_ptx.cuh",
                 os.path.join("..", "..", "include", "gg_backend.hpp")],
        "flags": ["-lcublas"],
    },
}


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    paths = [os.path.join(CSRC, d) for d in deps] + [os.path.join(INCLUDE, "gg_b200.h")]
    return any(os.path.exists(p) and os.path.getmtime(p) > t for p in paths)


def build(force: bool = False, verbose: bool = False) -> list[str]:
    os.makedirs(LIB, exist_ok=True)
    built = []
    for name, t in TARGETS.items():
        srcs = [os.path.join(CSRC, s) for s in t["srcs"]]
        if not all(os.path.exists(s) for s in srcs):
            continue
        out = os.path.join(LIB, name)
        if not force and not _stale(out, t["deps"]):
            continue
        cmd = [NVCC] + COMMON + t["flags"] + ["-o", out] + srcs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        built.append(out)
    return built


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose=True):
        print("built", p)
