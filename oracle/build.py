"""Build recipe for the test oracle (checker only, never shipped on the product path).

  lib/liboracle.so     CPU restatement (gg_oracle.cpp), g++
  _ref/ref_harness     the reference's own bench/bench_main.cpp (fill_randn, make_samples,
                       sampled_reference, check_output ...) compiled UNMODIFIED from the mounted
                       reference tree with nvcc, through the HIP->CUDA shim headers in ref_shim/,
                       and wrapped by ref_harness.cu. Built only where the reference tree exists;
                       the binary then travels with the snapshot.

Usage: python build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib")
REF_OUT = os.path.join(HERE, "_ref")
# The reference project's source tree: $GG_REFERENCE_ROOT, else a directory named `reference`
# beside this repository's root. Where neither exists the reference harness is not built.
REFERENCE = os.environ.get("GG_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build_oracle(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(LIB, exist_ok=True)
    src = os.path.join(HERE, "gg_oracle.cpp")
    out = os.path.join(LIB, "liboracle.so")
    if force or _stale(out, [src, __file__]):
        # x86-64-v3 = AVX2 + FMA: every B200 host has it.
        cmd = ["g++", "-O3", "-march=x86-64-v3", "-std=c++17", "-fPIC", "-shared", "-pthread",
               "-o", out, src]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return out


def build_ref_harness(force: bool = False, verbose: bool = False) -> str | None:
    bench_src = os.path.join(REFERENCE, "bench", "bench_main.cpp")
    if not os.path.exists(bench_src):
        return None  # GPU box: uses the prebuilt binary that travelled with the snapshot
    os.makedirs(REF_OUT, exist_ok=True)
    out = os.path.join(REF_OUT, "ref_harness")
    wrapper = os.path.join(HERE, "ref_harness.cu")
    shim = os.path.join(HERE, "ref_shim")
    deps = [wrapper, bench_src, os.path.join(REFERENCE, "common", "backend.hpp"), __file__,
            os.path.join(shim, "hip", "hip_runtime.h")]
    if force or _stale(out, deps):
        cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
               "-I" + shim, "-I" + os.path.join(REFERENCE, "common"), "-I" + REFERENCE,
               "-o", out, wrapper, "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return out


def build(force: bool = False, verbose: bool = False) -> None:
    build_oracle(force, verbose)
    build_ref_harness(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
