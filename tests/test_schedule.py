"""CPU: the kernel's work-unit schedule, walked on the host.

`tests/sched_check.cu` calls the kernel's own `units_of` / `unit_at` (host-callable in
gg_kernel.cuh) and the library's stream-K arithmetic (gg_sched.h) for every cluster of 20000
random launches of each schedule form (whole tiles, plain split-K, split-K of the partial last
wave, stream-K of kind 1 and 2). It checks that every (tile, K atom) is covered exactly once,
that a tile's pieces are numbered in K order (the fixed order the partial sums are added in),
that a tile in pieces has workspace, and that the stream-K summer only waits for pieces that
are the first unit of their cluster (no circular wait). It also walks the kernel's `decode_tile`
over random group tables (empty groups, both raster orders, every band) and checks that tile
indices cover every (group, m-tile, n-tile) exactly once. The GPU parity tests check the same
code through their results; this walks far more shapes than a GPU run can.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "groupgemm-cktile-optimized_b200", "csrc")


def _nvcc():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    return nvcc


def test_schedule_covers_every_atom_once_and_summer_never_waits_in_a_cycle(tmp_path):
    exe = tmp_path / "sched_check"
    build = subprocess.run([_nvcc(), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
                            "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-o", str(exe),
                            os.path.join(ROOT, "tests", "sched_check.cu")],
                           capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-2000:]
    run = subprocess.run([str(exe), "20000"], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout[-2000:] + run.stderr[-2000:]
    assert run.stdout.startswith("ok "), run.stdout
