"""CPU: `bench.py`'s host-side pieces.

* The reference arm (`--impl reference`: the oracle port of the reference's fp32 math on the host
  cores, the arm the driver runs beside this library's) prints one JSON line with the contract's
  keys, on rank 0 only.
* Config U's skewed routing is seeded (the same sizes every run), routes every token, and the
  sizes a rank takes for its expert shard are that shard's slice of the whole job's sizes.
"""
import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("gg_bench_driver", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, RANK="0")
    run = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert run.returncode == 0, run.stderr[-2000:]
    line = json.loads(run.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "TFLOPS"
    assert line["steps"] == 1 and line["warmup"] >= 3 and line["higher_is_better"] is True
    assert line["config"]["workload"].startswith("L:")
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_is_silent_on_other_ranks():
    env = dict(os.environ, RANK="1")
    run = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert run.returncode == 0, run.stderr[-2000:]
    assert run.stdout.strip() == ""


def test_skewed_routing_is_seeded_complete_and_shard_consistent():
    bench = _bench()
    cfg = bench.CONFIGS["U"]
    total, experts = cfg["m"] * cfg["b"], cfg["b"]
    whole = bench.group_sizes(cfg, 0, experts)
    assert whole == bench.group_sizes(cfg, 0, experts)  # seeded
    assert len(whole) == experts and sum(whole) == total and min(whole) >= 0
    assert max(whole) > 10 * (total // experts)  # skewed: one expert far above the mean
    for world in (2, 4, 8):
        parts = []
        for rank in range(world):
            g0 = rank * experts // world
            g1 = (rank + 1) * experts // world
            parts += bench.group_sizes(cfg, g0, g1)
        assert parts == whole
    balanced = bench.CONFIGS["E"]
    assert bench.group_sizes(balanced, 3, 7) == [balanced["m"]] * 4
