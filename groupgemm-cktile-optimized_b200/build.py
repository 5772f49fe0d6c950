"""Build recipe for the B200 grouped-GEMM library (nvcc, sm_100a only).

Outputs, in-tree so they travel with the repository snapshot:
  lib/libgg_b200.so   C ABI of include/gg_b200.h (static CUDA runtime)
  lib/libgg_b200_debug.so  the same with the kernel's bounds checks (-DGG_DEBUG)
  lib/gg_bench        C++ shapes-CSV -> results-CSV benchmark (bench_main contract)

Usage: python build.py [--force] [--resource-usage]

--resource-usage recompiles the library with `-Xptxas -v` and prints, per kernel instantiation,
registers per thread, spill stores/loads, stack frame and barriers (the counterpart of the
reference's -Rpass-analysis=kernel-resource-usage build flag, CMakeLists.txt:36-37).
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
import tempfile

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
        "deps": ["gg_capi.cu", "gg_kernel.cuh", "gg_ptx.cuh", "gg_sched.h"],
        "flags": ["-Xcompiler", "-fPIC", "-shared"],
    },
    # the same library with the kernel's bounds checks compiled in (-DGG_DEBUG): a failed check
    # records its site in the device status word and skips the access
    "libgg_b200_debug.so": {
        "srcs": ["gg_capi.cu"],
        "deps": ["gg_capi.cu", "gg_kernel.cuh", "gg_ptx.cuh", "gg_sched.h"],
        "flags": ["-Xcompiler", "-fPIC", "-shared", "-DGG_DEBUG"],
    },
    "gg_bench": {
        "srcs": ["gg_bench_main.cu", "gg_cublas_backends.cpp", "gg_capi.cu"],
        "deps": ["gg_bench_main.cu", "gg_cublas_backends.cpp", "gg_capi.cu", "gg_kernel.cuh", "gg_ptx.cuh", "gg_sched.h",
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


_OP = {"0": "forward", "1": "dgrad", "2": "wgrad"}


def _kernel_name(mangled: str) -> str:
    """Readable name of a grouped_gemm_sm100<T, kCG, kBN, kAtoms, kOp> instantiation."""
    m = re.search(r"grouped_gemm_sm100I(6__half|13__nv_bfloat16)Li(\d+)ELi(\d+)ELi(\d+)ELi(\d+)E", mangled)
    if not m:
        return re.sub(r"^_ZN.*?\d+([a-z_]+)E.*$", r"\1", mangled)
    dt = "fp16" if m.group(1) == "6__half" else "bf16"
    return f"grouped_gemm_sm100<{dt}, cta_group={m.group(2)}, BN={m.group(3)}, atoms={m.group(4)}, {_OP[m.group(5)]}>"


def resource_usage() -> list[dict]:
    """Compile the library with -Xptxas -v into a scratch file; one row per kernel."""
    with tempfile.TemporaryDirectory() as d:
        cmd = [NVCC] + COMMON + TARGETS["libgg_b200.so"]["flags"] + ["-Xptxas", "-v", "-o",
                                                                     os.path.join(d, "libgg_b200.so"),
                                                                     os.path.join(CSRC, "gg_capi.cu")]
        run = subprocess.run(cmd, check=True, capture_output=True, text=True)
    rows, cur = [], None
    for line in (run.stdout + run.stderr).splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = {"kernel": _kernel_name(m.group(1))}
            rows.append(cur)
            continue
        if cur is None:
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and "stack" not in cur:
            cur.update(stack=int(m.group(1)), spill_st=int(m.group(2)), spill_ld=int(m.group(3)))
        m = re.search(r"Used (\d+) registers, used (\d+) barriers", line)
        if m:
            cur.update(regs=int(m.group(1)), barriers=int(m.group(2)))
    return rows


if __name__ == "__main__":
    if "--resource-usage" in sys.argv:
        print("| kernel | registers | spill stores (B) | spill loads (B) | stack (B) | barriers |")
        print("|---|---:|---:|---:|---:|---:|")
        for r in sorted(resource_usage(), key=lambda r: r["kernel"]):
            print(f"| `{r['kernel']}` | {r.get('regs')} | {r.get('spill_st')} | {r.get('spill_ld')} | "
                  f"{r.get('stack')} | {r.get('barriers')} |")
    else:
        for p in build(force="--force" in sys.argv, verbose=True):
            print("built", p)
