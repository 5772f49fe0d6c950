"""The C++ harness gg_bench keeps the reference's command line and CSV contract
(bench/bench_main.cpp of the reference). CPU tests cover the argument handling (parsing happens
before any CUDA call); the GPU test runs the harness end to end on small shapes with b200 knobs
passed through --opt and checks every row of its results CSV."""
import csv
import os
import subprocess

import pytest

from conftest import ROOT

BIN = os.path.join(ROOT, "groupgemm-cktile-optimized_b200", "lib", "gg_bench")
SHAPES = os.path.join(ROOT, "groupgemm-cktile-optimized_b200", "shapes", "pad.csv")


def run(*args, timeout=120):
    return subprocess.run([BIN, *args], capture_output=True, text=True, timeout=timeout)


def test_binary_built():
    assert os.access(BIN, os.X_OK), "build gg_bench with groupgemm-cktile-optimized_b200/build.py"


@pytest.mark.parametrize("args,msg", [
    (["--help"], "usage: gg_bench"),
    ([], "--shapes is required"),
    (["--shapes", SHAPES, "--opt", "variant"], "--opt wants KEY=VALUE"),
    (["--shapes", SHAPES, "--opt", "bn=abc"], "not an integer"),
    (["--shapes", SHAPES, "--dtype", "fp8"], "--dtype must be bf16 or fp16"),
    (["--shapes", SHAPES, "--iters", "0"], "--iters must be >= 1"),
    (["--shapes", SHAPES, "--bogus"], "unknown argument --bogus"),
])
def test_usage_errors(args, msg):
    r = run(*args)
    assert r.returncode == 2, (r.returncode, r.stderr)
    assert msg in r.stderr, r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("opts", [[], ["--opt", "store=0"], ["--opt", "variant=1", "--opt", "store=1"]])
def test_harness_runs_and_checks(tmp_path, opts):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    out = tmp_path / "results.csv"
    r = run("--shapes", SHAPES, "--backends", "b200", "--only", "9002,9003,9101,9102", "--warmup", "1", "--iters", "2",
            "--out", str(out), *opts)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    rows = list(csv.DictReader(open(out)))
    assert len(rows) == 4
    for row in rows:
        assert row["Backend"] == "b200" and row["Check"] == "PASS", row
        assert float(row["TFLOPS"]) > 0
    if "variant=1" in opts:
        assert all("cta_group=1" in row["Detail"] for row in rows), [row["Detail"] for row in rows]
