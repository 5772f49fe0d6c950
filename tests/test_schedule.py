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


@pytest.fixture(scope="module")
def sched_check(tmp_path_factory):
    exe = tmp_path_factory.mktemp("sched") / "sched_check"
    build = subprocess.run([_nvcc(), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
                            "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-o", str(exe),
                            os.path.join(ROOT, "tests", "sched_check.cu")],
                           capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-2000:]
    return str(exe)


def test_schedule_covers_every_atom_once_and_summer_never_waits_in_a_cycle(sched_check):
    run = subprocess.run([sched_check, "20000"], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout[-2000:] + run.stderr[-2000:]
    assert run.stdout.startswith("ok "), run.stdout


# The cost model's automatic choices on the BASELINE shapes, each the measured best of the
# alternatives tried on a B200 (interleaved A/B runs): pair 256 x 256 tiles for L, D and E, pair
# 256 x 240 for P (12 x 240 = 2880, no N padding), one wave of 144 one-CTA 128 x 160 tiles for the
# B=1 variant of P, one-CTA 128 x 96 tiles for T, 256 x 256 with the partial last wave split 3
# ways in K for W, and one wave of 70 pairs of 256 x 176 tiles for the suite's single-expert
# 1 x 512 x 6144 x 16384 (+5.5% over 3-way split-K). A model change that moves one of these must
# come with new measurements.
PINNED = {
    "8,4096,4096,7168": (0, 256, 1, 0, 0),     # L
    "32,2048,7168,2048": (0, 256, 1, 0, 0),    # D
    "256,512,4096,7168": (0, 256, 1, 0, 0),    # E
    "16,1000,2880,2880": (0, 240, 1, 0, 0),    # P
    "1,1000,2880,2880": (1, 160, 1, 0, 0),     # P, B=1
    "4,256,512,384": (2, 96, 1, 0, 0),         # T
    "2,512,6144,8192": (0, 256, 3, 1, 0),      # W (last-wave split)
    "1,512,6144,16384": (0, 176, 1, 0, 0),     # suite TestID 278: one wave of 70 pairs, no split
}


def _choose(exe, shapes):
    run = subprocess.run([exe, "choose", *shapes], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    return [tuple(int(v) for v in line.split()) for line in run.stdout.split("\n") if line.strip()]


def test_cost_model_keeps_the_measured_best_choices(sched_check):
    got = _choose(sched_check, list(PINNED))
    assert dict(zip(PINNED, got)) == PINNED


def test_cost_model_width_rules_hold_on_many_shapes(sched_check):
    # widths in steps of 16; a width that is not a multiple of 32 only where it tiles N exactly
    # or, at 160 columns or more, fits the launch in one wave; below 128 columns only when the
    # tiling fits in one wave; stream-K never by default
    import itertools
    shapes = [f"{b},{m},{n},{k}" for b, m, n, k in itertools.product(
        (1, 2, 4, 8, 16, 64), (256, 512, 1000, 2048, 8192), (512, 1536, 2816, 2880, 4096, 5760, 7168),
        (384, 2048, 2880, 7168))]
    for shape, (variant, bn, splits, hybrid, sk) in zip(shapes, _choose(sched_check, shapes)):
        b, m, n, k = (int(v) for v in shape.split(","))
        assert bn % 16 == 0 and sk == 0, shape
        cluster_m = 256 if variant == 0 else 128
        slots = 74 if variant == 0 else 148
        one_wave = b * -(-m // cluster_m) * -(-n // bn) <= slots
        if bn % 32:
            assert n % bn == 0 or (bn >= 160 and one_wave), shape
        if bn < 128:
            assert one_wave, shape
