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


def test_roofline_traffic_follows_the_shard_and_stays_under_hbm_peak():
    """The DRAM traffic a rank's roofline reports is its own launch's: a capture of the same size
    is used as is, another size is scaled by the algorithmic bytes, so the traffic rate of a
    shard never reads above the measured copy bandwidth (a shard's launch time shrinks with its
    bytes). Launch times here come from a fixed per-GPU rate (1400 TFLOPS), as a bench would see."""
    bench = _bench()
    peaks = {"bf16_tflops": 1690.7, "bf16_tflops_sustained": 1409.9, "hbm_gbs": 6540.8}
    for name in ("E", "L"):
        cfg = bench.CONFIGS[name]
        caps = bench.load_traffic(name)
        assert caps and all(c["algorithmic_bytes"] > 0 for c in caps), name
        for world in (1, 2, 4, 8):
            total = cfg["b"] * world if cfg["per_gpu"] else cfg["b"]
            for rank in (0, world - 1):
                g0, g1 = rank * total // world, (rank + 1) * total // world
                gm = bench.group_sizes(cfg, g0, g1)
                alg = bench.algorithmic_bytes(gm, cfg["n"], cfg["k"])
                flops = 2.0 * sum(gm) * cfg["n"] * cfg["k"]
                ms = flops / 1400e12 * 1e3
                r = bench.roofline(flops, alg, ms, peaks, "measured", caps, "test")
                assert r["traffic"] is not None and r["traffic"] >= 0.99 * alg, (name, world, r)
                assert r["hbm"]["traffic_gbs"] < r["hbm"]["peak_gbs"], (name, world, r["hbm"])
                exact = any(c["algorithmic_bytes"] == alg for c in caps)
                assert ("scaled" in r["traffic_source"]) == (not exact), (name, world, r["traffic_source"])
    # no capture: null traffic with a reason, never a number from another launch
    r = bench.roofline(1e12, 1e9, 1.0, peaks, "measured", [], "test")
    assert r["traffic"] is None and r["hbm"]["traffic_gbs"] is None and r["traffic_source"]


def test_reference_arm_and_cpu_baseline_time_the_same_unit(monkeypatch):
    """Both CPU figures are whole experts of the workload on all host threads (one expert per
    step in the reference arm), so they measure the same thing."""
    bench = _bench()
    calls = []

    class FakeOracle:
        @staticmethod
        def hw_threads():
            return 4

        @staticmethod
        def make_inputs(group_m, n, k, dt):
            return None, None

        @staticmethod
        def grouped_gemm_f32(x, w, group_m, dt, threads=0, out=None, **kw):
            calls.append((tuple(group_m), kw.get("max_rows", -1), None if out is None else out.shape))

    monkeypatch.setattr(bench, "load_oracle", lambda: FakeOracle)
    cfg = dict(bench.CONFIGS["L"], m=64, n=32, k=16)
    bench.cpu_baseline(cfg, budget_s=60)
    base_calls, calls[:] = list(calls), []

    class Args:
        steps, warmup, gpus = 2, 3, 1

    monkeypatch.setenv("RANK", "0")
    bench.run_reference(Args, cfg)
    assert base_calls and calls and set(base_calls) == set(calls) == {((64,), -1, (64, 32))}
    assert len(calls) == Args.steps + Args.warmup
