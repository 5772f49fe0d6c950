"""Benchmark of the B200 grouped GEMM (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config L|E|...]

Workload ("L"): a balanced MoE gate/up projection, B=8 experts per GPU,
M=4096 tokens per expert, N=4096, K=7168, bf16 in / fp32 accumulate / bf16 out. Inputs are
N(0,1), generated on the device (bf16), 940 MB per GPU, larger than the 126 MB L2, so no L2
flush is needed between steps. A step is one grouped GEMM over all of the GPU's experts,
enqueued through the C ABI (gg_run), timed back to back like the reference harness
(bench/bench_main.cpp:490-501).

Multi-GPU (torchrun, one process per GPU, NCCL only for the barrier and the max-over-ranks
timing): experts are sharded contiguously (gg_expert_shard); every GPU keeps 8 experts of L, so
the job grows with N ("scaling": "weak"). There is no collective on the GEMM path. Beside it, at
every N, the same line carries `config_E`: BASELINE configs[4] (256 experts in total) sharded
over the N GPUs (strong scaling), with rank 0's one-GPU time of the whole problem in the same run
as the efficiency base, and (with --allgather) an NCCL all-gather of its outputs, timed apart.
After the timed region a seconds-long back-to-back leg on the headline config reports the
sustained (power-capped) throughput and SM clock (`sustained`).

`--impl reference` times the reference op's CPU fp32 path (the reference has no CPU
implementation; the oracle port of its fp32 math runs on all host cores), one whole expert of
the workload per step, on rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "groupgemm-cktile-optimized_b200")

METRIC = "grouped-GEMM TFLOPS/GPU (bf16) and % of B200 dense peak; aggregate at 1/2/4/8 GPU"
DATASHEET_TFLOPS = 2250.0
FALLBACK = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}

CONFIGS = {
    # name: (experts per GPU or total, M, N, K, dtype, sharding)
    "L": dict(b=8, m=4096, n=4096, k=7168, dtype="bf16", per_gpu=True,
              desc="L: B=8 experts per GPU, M=4096, N=4096, K=7168, bf16 (BASELINE configs[1])"),
    "E": dict(b=256, m=512, n=4096, k=7168, dtype="bf16", per_gpu=False,
              desc="E: B=256 experts sharded over the GPUs, M=512, N=4096, K=7168, bf16 (BASELINE configs[4])"),
    # E's per-GPU share at 8 GPUs on its own (the reduced case for DRAM captures)
    "E32": dict(b=32, m=512, n=4096, k=7168, dtype="bf16", per_gpu=True,
                desc="E32: config E's per-GPU share at 8 GPUs, B=32 experts, M=512, N=4096, K=7168, bf16"),
    "D": dict(b=32, m=2048, n=7168, k=2048, dtype="fp16", per_gpu=True,
              desc="D: B=32 experts per GPU, M=2048, N=7168, K=2048, fp16 (BASELINE configs[2])"),
    "P": dict(b=16, m=1000, n=2880, k=2880, dtype="bf16", per_gpu=True,
              desc="P: B=16 experts per GPU, M=1000, N=2880, K=2880, bf16 (BASELINE configs[3])"),
    "P1": dict(b=1, m=1000, n=2880, k=2880, dtype="bf16", per_gpu=True,
               desc="P1: B=1 expert, M=1000, N=2880, K=2880, bf16 (BASELINE configs[3], B=1 variant: low tile count)"),
    # synthetic: 2 x 2 x 24 = 96 pair tiles for 74 CTA pairs, a partial last wave (split-K of the
    # last wave only)
    "W": dict(b=2, m=512, n=6144, k=8192, dtype="bf16", per_gpu=True,
              desc="W: synthetic B=2, M=512, N=6144, K=8192, bf16 (96 pair tiles on 74 pairs: a partial last wave)"),
    "T": dict(b=4, m=256, n=512, k=384, dtype="bf16", per_gpu=True,
              desc="T: B=4, M=256, N=512, K=384, bf16 (BASELINE configs[0])"),
    # E's 131072 tokens routed unevenly (Zipf-like expert popularity, seeded), some experts empty
    "U": dict(b=256, m=512, n=4096, k=7168, dtype="bf16", per_gpu=False, skew=1.1,
              desc="U: config E with 131072 tokens over 256 experts routed with Zipf(1.1) popularity (seeded)"),
}


def group_sizes(cfg, g0, g1):
    """Rows per expert of experts [g0, g1): balanced, or the seeded skewed routing of config U."""
    if "skew" not in cfg:
        return [cfg["m"]] * (g1 - g0)
    total, experts = cfg["m"] * cfg["b"], cfg["b"]
    rng = np.random.default_rng(2024)
    weights = 1.0 / np.arange(1, experts + 1) ** cfg["skew"]
    weights = weights[rng.permutation(experts)]
    sizes = np.floor(weights / weights.sum() * total).astype(np.int64)
    sizes[np.argmax(sizes)] += total - sizes.sum()
    return [int(v) for v in sizes[g0:g1]]


def algorithmic_bytes(group_m, n, k, elem=2):
    """Each operand read once, the output written once: 2 (sum(M) K + B N K + sum(M) N)."""
    rows = int(sum(group_m))
    return int(elem * (rows * k + len(group_m) * n * k + rows * n))


def load_package():
    spec = importlib.util.spec_from_file_location("gg_b200", os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["gg_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    """CPU oracle: only the CPU-baseline leg and the reference arm use it."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402

    return oracle


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK), "fallback"


def shard_of(cfg, world, rank, gg):
    """(global group count, [g0, g1) of this rank)."""
    total = cfg["b"] * world if cfg["per_gpu"] else cfg["b"]
    return total, gg.expert_shard(total, world, rank)


class ClockSampler:
    """Samples SM clock, power draw and clock-event reasons through NVML (read-only) every ~5 ms."""

    REASONS = {
        "gpu_idle": "nvmlClocksEventReasonGpuIdle",
        "applications_clocks_setting": "nvmlClocksEventReasonApplicationsClocksSetting",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "sync_boost": "nvmlClocksEventReasonSyncBoost",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
        "display_clock_setting": "nvmlClocksEventReasonDisplayClockSetting",
    }

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.power_w = [], set(), []
        self.mask = 0
        self.max_mhz = None
        self.power_limit_w = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            try:
                self.power_limit_w = pynvml.nvmlDeviceGetEnforcedPowerLimit(self._h) / 1000.0
            except Exception:
                pass
        except Exception as e:  # NVML missing: report no clocks rather than fail the bench
            self._nv = None
            self.error = str(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.mask |= int(r)
                for name, attr in self.REASONS.items():
                    if r & getattr(nv, attr, 0):
                        self.reasons.add(name)
                self.power_w.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self):
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.samples),
               "reason_mask": hex(self.mask)}
        if self.power_w:
            out["power_w_max"] = round(max(self.power_w), 1)
            out["power_w_median"] = round(statistics.median(self.power_w), 1)
        if self.power_limit_w:
            out["power_limit_w"] = self.power_limit_w
        return out


def cpu_expert_rate(cfg, orc, threads, x, w, steps):
    """Seconds of each of `steps` whole-expert fp32 GEMMs (M x N x K) with the oracle port."""
    dt = 0 if cfg["dtype"] == "bf16" else 1
    out = np.zeros((cfg["m"], cfg["n"]), np.float32)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        orc.grouped_gemm_f32(x, w, [cfg["m"]], dt, threads=threads, out=out)
        times.append(time.perf_counter() - t0)
    return times


def cpu_baseline(cfg, budget_s: float = 20.0):
    """Oracle port of the fp32 reference path on all host cores. Whole experts of the workload
    (M x N x K each) are computed one after another until every expert of one GPU's share is
    done or `budget_s` has passed; the sample is the experts completed. The reference arm
    (`--impl reference`) times the same unit, one expert per step."""
    orc = load_oracle()
    dt = 0 if cfg["dtype"] == "bf16" else 1
    n, k, m, b = cfg["n"], cfg["k"], cfg["m"], cfg["b"]
    threads = orc.hw_threads()
    x, w = orc.make_inputs([m], n, k, dt)  # one expert's operands, reused per expert
    done, el = 0, 0.0
    while done < b and el < budget_s:
        el += cpu_expert_rate(cfg, orc, threads, x, w, 1)[0]
        done += 1
    flops = 2.0 * done * m * n * k
    return {"value": round(flops / el / 1e12, 4), "unit": "TFLOPS", "cores": threads, "kind": "port",
            "sample": f"{done} of {b} experts of the workload (each fp32 {m}x{n}x{k}; {flops / 1e9:.0f} GFLOP, "
                      f"{el:.2f} s) with the oracle port on {threads} host threads"}


def run_reference(args, cfg):
    """The reference arm: the oracle port of the reference op's fp32 math (the reference has no
    CPU implementation of its own) on all host threads. A step is one whole expert of the
    workload (M x N x K), the unit `cpu_baseline` times too."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    orc = load_oracle()
    dt = 0 if cfg["dtype"] == "bf16" else 1
    n, k, m = cfg["n"], cfg["k"], cfg["m"]
    threads = orc.hw_threads()
    x, w = orc.make_inputs([m], n, k, dt)
    cpu_expert_rate(cfg, orc, threads, x, w, args.warmup)
    times = cpu_expert_rate(cfg, orc, threads, x, w, args.steps)
    el = sum(times)
    flops = 2.0 * m * n * k * args.steps
    value = flops / el / 1e12
    sample = (f"each step: fp32 GEMM of one whole expert ({m} rows x N={n} x K={k}) of the {cfg['desc']} workload, "
              f"oracle port of the reference's fp32 math on {threads} host threads")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "TFLOPS", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * el / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic N(0,1), reference generator",
        "config": {"workload": cfg["desc"], "global_batch": cfg["b"] * cfg["m"], "parallelism": "cpu"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def load_traffic(cfg_name):
    """ncu DRAM captures of the kernel for a config (profiles/gg_sm100_<cfg>_traffic.json): a list
    of {bytes_per_launch, algorithmic_bytes, source, ...}, one per captured launch size."""
    path = os.path.join(ROOT, "profiles", f"gg_sm100_{cfg_name}_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return []
    caps = d.get("captures", [d]) if isinstance(d, dict) else d
    return [c for c in caps if c.get("bytes_per_launch")]


def launch_traffic(captures, alg_bytes):
    """DRAM bytes of one launch whose algorithmic bytes are `alg_bytes`, from the captures of the
    same config: the capture of that size if there is one, else the capture nearest in size with
    its traffic scaled in proportion to the algorithmic bytes (the re-read factor is taken as
    size-independent, which the source string says). (None, reason) when nothing applies."""
    usable = [c for c in captures if c.get("algorithmic_bytes")]
    if not usable:
        return None, "no ncu DRAM capture with its algorithmic bytes for this config"
    best = min(usable, key=lambda c: abs(np.log(c["algorithmic_bytes"] / alg_bytes)))
    if best["algorithmic_bytes"] == alg_bytes:
        return int(best["bytes_per_launch"]), best.get("source", "")
    scaled = int(round(best["bytes_per_launch"] * alg_bytes / best["algorithmic_bytes"]))
    ratio = best["bytes_per_launch"] / best["algorithmic_bytes"]
    return scaled, (f"scaled from a capture of {best['algorithmic_bytes'] / 1e9:.3f} GB algorithmic "
                    f"({ratio:.3f}x traffic/algorithmic) to this launch's {alg_bytes / 1e9:.3f} GB: "
                    f"{best.get('source', '')}")


def roofline(flops, alg_bytes, ms_launch, peaks, peak_src, captures, kernel_detail):
    """Roofline object of one rank's launch: tensor side against the measured cuBLAS burst, memory
    side (algorithmic bytes and ncu DRAM traffic, scaled to this launch) against the measured copy
    bandwidth."""
    achieved = flops / (ms_launch * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK["bf16_tflops"]))
    sustained_peak = float(peaks.get("bf16_tflops_sustained", FALLBACK["bf16_tflops_sustained"]))
    traffic, tsrc = launch_traffic(captures, alg_bytes)
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK["hbm_gbs"]))
    alg_gbs = alg_bytes / (ms_launch * 1e-3) / 1e9
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} bf16 burst (cuBLAS)",
            "frac_of_sustained": round(achieved / sustained_peak, 4),
            "frac_of_datasheet_2250": round(achieved / DATASHEET_TFLOPS, 4),
            "traffic": traffic, "traffic_source": tsrc, "algorithmic_bytes": int(alg_bytes),
            "kernel": "gg::grouped_gemm_sm100 (" + kernel_detail + ")",
            "hbm": {"algorithmic_gbs": round(alg_gbs, 1), "peak_gbs": hbm_peak,
                    "frac_algorithmic": round(alg_gbs / hbm_peak, 4),
                    "traffic_gbs": round(traffic / (ms_launch * 1e-3) / 1e9, 1) if traffic else None}}


def run_vs_loop(args, cfg):
    """One grouped GEMM (forward, dgrad or wgrad) on one GPU beside a per-group cuBLAS loop
    (torch.matmul, one stream) of the same op on the same tensors. The two arms alternate in
    rounds of a few steps each, so both see the same clocks and power state (at the 1000 W cap the
    clock moves by 30% within seconds); each arm's figure is its median round. One JSON line; not
    the driver's headline (that is the forward op through the full bench line)."""
    import statistics

    import torch

    gg = load_package()
    op = {"forward": gg.OP_FORWARD, "dgrad": gg.OP_DGRAD, "wgrad": gg.OP_WGRAD}[args.op]
    dtype = gg.DTYPES[cfg["dtype"]]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    torch.cuda.set_device(0)
    total_groups, (g0, g1) = shard_of(cfg, 1, 0, gg)
    ng = g1 - g0
    n, k = cfg["n"], cfg["k"]
    group_m = group_sizes(cfg, g0, g1)
    rows = sum(group_m)
    gen = torch.Generator(device="cuda").manual_seed(1000)

    def randn(*shape):
        return torch.randn(*shape, device="cuda", generator=gen, dtype=torch.float32).to(tdt)

    def weights():
        w = torch.empty(ng, n, k, device="cuda", dtype=tdt)
        for g in range(ng):
            w[g] = randn(n, k)
        return w

    if op == gg.OP_FORWARD:
        a_op, b_op = randn(rows, k), weights()
        out = torch.empty(rows, n, device="cuda", dtype=tdt)
    elif op == gg.OP_DGRAD:
        a_op, b_op = randn(rows, n), weights()
        out = torch.empty(rows, k, device="cuda", dtype=tdt)
    else:
        a_op, b_op = randn(rows, n), randn(rows, k)
        out = torch.empty(ng, n, k, device="cuda", dtype=tdt)
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    be = gg.make_b200_backend()
    if args.variant >= 0:
        be.set_option("variant", args.variant)
    for kv in args.opt:
        key, _, val = kv.partition("=")
        be.set_option(key, int(val))
    if op == gg.OP_FORWARD:
        why = be.prepare(dtype, group_m, n, k, a_op.data_ptr(), b_op.data_ptr(), out.data_ptr(), s)
    elif op == gg.OP_DGRAD:
        why = be.prepare_grad(op, dtype, group_m, n, k, dy_ptr=a_op.data_ptr(), w_ptr=b_op.data_ptr(),
                              dx_ptr=out.data_ptr(), stream=s)
    else:
        why = be.prepare_grad(op, dtype, group_m, n, k, dy_ptr=a_op.data_ptr(), x_ptr=b_op.data_ptr(),
                              dw_ptr=out.data_ptr(), stream=s)
    if why:
        raise SystemExit(f"prepare refused the workload: {why}")
    offs = np.concatenate([[0], np.cumsum(group_m)]).tolist()

    def cublas_step(dst):
        for g in range(ng):
            a, b = offs[g], offs[g + 1]
            if op == gg.OP_FORWARD:
                if b > a:
                    torch.matmul(a_op[a:b], b_op[g].t(), out=dst[a:b])
            elif op == gg.OP_DGRAD:
                if b > a:
                    torch.matmul(a_op[a:b], b_op[g], out=dst[a:b])
            elif b > a:
                torch.matmul(a_op[a:b].t(), b_op[a:b], out=dst[g])
            else:
                dst[g].zero_()  # an expert without tokens: dw[g] = 0, as the kernel writes

    ref = torch.empty_like(out)
    # The loop is replayed from a CUDA graph, so its hundreds of small launches per step cost no
    # host time (issued from Python one by one they can leave the GPU idle between experts).
    with torch.cuda.stream(stream):
        cublas_step(ref)  # cuBLAS workspace and handles before capture
    torch.cuda.synchronize()
    loop_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(loop_graph, stream=torch.cuda.Stream()):
        cublas_step(ref)

    def loop_replay():
        loop_graph.replay()

    arms = {"ours": lambda: be.run(s), "loop": loop_replay}
    rounds = 5
    per_round = max(2, args.steps // rounds)
    ms_rounds = {a: [] for a in arms}
    with torch.cuda.stream(stream):
        for fn in arms.values():
            for _ in range(args.warmup):
                fn()
    torch.cuda.synchronize()
    with ClockSampler(0) as clocks:
        for _ in range(rounds):
            for a, fn in arms.items():
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    ev0.record(stream)
                    for _ in range(per_round):
                        fn()
                    ev1.record(stream)
                ev1.synchronize()
                ms_rounds[a].append(ev0.elapsed_time(ev1) / per_round)
    if be.device_status(s) != 0:
        raise SystemExit("kernel reported a bounded-wait timeout")
    ms, ms_cublas = statistics.median(ms_rounds["ours"]), statistics.median(ms_rounds["loop"])
    # check against cuBLAS on the same tensors: the reference pass rule on every element checked
    with torch.cuda.stream(stream):
        be.run(s)
        ref.zero_()
        loop_replay()
    torch.cuda.synchronize()
    del loop_graph
    lim = min(out.numel(), 1 << 26)  # the first 64M elements (bounded temporaries)
    o32, r32 = out.view(-1)[:lim].float(), ref.view(-1)[:lim].float()
    diff = (o32 - r32).abs()
    bad = int((diff > 1e-2 + 2e-2 * r32.abs()).sum().item())
    flops = 2.0 * rows * n * k
    value = flops / (ms * 1e-3) / 1e12
    peaks, peak_src = measured_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK["bf16_tflops"]))
    what = {gg.OP_FORWARD: "out = x[g] @ w[g]^T", gg.OP_DGRAD: "dx = dy @ w[g]", gg.OP_WGRAD: "dw[g] = dy[g]^T @ x[g]"}
    line = {
        "metric": f"grouped-GEMM TFLOPS/GPU ({cfg['dtype']}), {args.op} beside a per-expert cuBLAS loop",
        "op": args.op, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": 1,
        "steps": rounds * per_round, "warmup": args.warmup, "rounds": rounds,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": cfg["dtype"],
        "data": "synthetic N(0,1) (torch generator on the device)",
        "config": {"workload": cfg["desc"], "op": what[op],
                   "l2": "inputs larger than L2 (no flush)" if rows * (n + k) * 2 > 126e6 else "inputs may fit in L2"},
        "roofline": {"bound": "tensor", "achieved": round(value, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(value / peak, 4), "peak_source": f"{peak_src} bf16 burst (cuBLAS)"},
        "cublas_loop": {"value": round(flops / (ms_cublas * 1e-3) / 1e12, 2), "unit": "TFLOPS",
                        "ms_per_step": round(ms_cublas, 4),
                        "how": "torch.matmul per expert, one stream, replayed from a CUDA graph"},
        "ratio_vs_loop": round(ms_cublas / ms, 3),
        "rounds_tflops": {a: [round(flops / (v * 1e-3) / 1e12) for v in ms_rounds[a]] for a in arms},
        "check_vs_cublas": {"elements": int(lim), "outside_tolerance": bad,
                            "max_abs_diff": float(diff.max().item())},
        "gpu_launches": rounds * per_round, "clocks": clocks.summary(), "detail": be.detail(),
    }
    be.release()
    print(json.dumps(line), flush=True)
    return 0 if bad == 0 else 1


class Problem:
    """One rank's share of a config on its GPU: seeded N(0,1) inputs generated on the device, the
    output buffer and a prepared backend handle."""

    def __init__(self, gg, torch, cfg, g0, g1, seed, stream, variant=-1, opts=()):
        self.cfg = cfg
        self.group_m = group_sizes(cfg, g0, g1)
        self.rows = sum(self.group_m)
        n, k = cfg["n"], cfg["k"]
        tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
        gen = torch.Generator(device="cuda").manual_seed(seed)
        self.x = torch.randn(self.rows, k, device="cuda", generator=gen, dtype=torch.float32).to(tdt)
        self.w = torch.empty(g1 - g0, n, k, device="cuda", dtype=tdt)
        for g in range(g1 - g0):  # per expert to bound the fp32 temporary
            self.w[g] = torch.randn(n, k, device="cuda", generator=gen, dtype=torch.float32).to(tdt)
        self.out = torch.empty(self.rows, n, device="cuda", dtype=tdt)
        self.flops = 2.0 * self.rows * n * k
        self.alg_bytes = algorithmic_bytes(self.group_m, n, k)
        self.backend = gg.make_b200_backend()
        self.opts = [("variant", variant)] if variant >= 0 else []
        self.opts += list(opts)
        for key, val in self.opts:
            self.backend.set_option(key, val)
        why = self.backend.prepare(gg.DTYPES[cfg["dtype"]], self.group_m, n, k, self.x.data_ptr(),
                                   self.w.data_ptr(), self.out.data_ptr(), stream.cuda_stream)
        if why:
            raise SystemExit(f"prepare refused the workload: {why}")

    def release(self):
        self.backend.release()
        del self.x, self.w, self.out


def time_launches(torch, prob, stream, steps, warmup, dist=None, sampler=None):
    """Mean device time (ms) of `steps` back-to-back launches after `warmup` untimed ones, CUDA
    events on the launching stream, barrier + synchronize on both sides. Returns (this rank's ms,
    max over ranks)."""
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            prob.backend.run(s)
    torch.cuda.synchronize()
    if prob.backend.device_status(s) != 0:
        raise SystemExit("kernel reported a bounded-wait timeout during warm-up")
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.__enter__()
    try:
        ev0.record(stream)
        for _ in range(steps):
            prob.backend.run(s)
        ev1.record(stream)
        ev1.synchronize()
    finally:
        if sampler:
            sampler.__exit__()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if prob.backend.device_status(s) != 0:
        raise SystemExit("kernel reported a bounded-wait timeout in a timed region")
    ms = ev0.elapsed_time(ev1) / steps
    return ms, max_over_ranks(torch, dist, ms)


def max_over_ranks(torch, dist, v):
    if not dist:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sustained_leg(torch, prob, stream, dist, local_rank, seconds, peaks):
    """Back-to-back launches for about `seconds` after the timed region: the throughput and SM
    clock the kernel holds once the board sits at its power cap."""
    s = stream.cuda_stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    prob.backend.run(s)
    ev1.record(stream)
    ev1.synchronize()
    launches = max(10, int(seconds * 1e3 / max(ev0.elapsed_time(ev1), 1e-3)))
    launches = int(max_over_ranks(torch, dist, launches))  # every rank runs the same count
    sampler = ClockSampler(local_rank)
    ms_rank, ms = time_launches(torch, prob, stream, launches, 0, dist, sampler)
    tflops = prob.flops / (ms_rank * 1e-3) / 1e12
    clk = sampler.summary()
    out = {"tflops_per_gpu": round(prob.flops / (ms * 1e-3) / 1e12, 2), "launches": launches,
           "seconds": round(ms * launches / 1e3, 2), "ms_per_launch": round(ms, 4),
           "median_sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons"),
           "power_w_median": clk.get("power_w_median"),
           "frac_of_sustained_peak": round(tflops / float(peaks.get("bf16_tflops_sustained",
                                                                    FALLBACK["bf16_tflops_sustained"])), 4),
           "frac_of_datasheet_2250": round(tflops / DATASHEET_TFLOPS, 4)}
    if clk.get("sm_mhz"):
        out["tflops_per_ghz"] = round(tflops / (clk["sm_mhz"] / 1e3), 1)
    return out


def config_e_leg(torch, gg, dist, world, rank, local_rank, stream, steps, warmup, allgather, peaks, peak_src):
    """BASELINE configs[4] (256 experts) sharded contiguously over the `world` GPUs: aggregate
    TFLOPS at max-over-ranks time, per-GPU TFLOPS, and the efficiency against rank 0's one-GPU
    time of the whole problem measured in the same run (the other ranks wait meanwhile)."""
    cfg = CONFIGS["E"]
    total_flops = 2.0 * sum(group_sizes(cfg, 0, cfg["b"])) * cfg["n"] * cfg["k"]
    ms_one = None
    if world > 1:
        if rank == 0:
            whole = Problem(gg, torch, cfg, 0, cfg["b"], 2000, stream)
            ms_one, _ = time_launches(torch, whole, stream, steps, warmup, None, ClockSampler(local_rank))
            whole.release()
            del whole
            torch.cuda.empty_cache()
        dist.barrier()
    g0, g1 = gg.expert_shard(cfg["b"], world, rank)
    prob = Problem(gg, torch, cfg, g0, g1, 2000 + rank, stream)
    clocks = ClockSampler(local_rank)
    ms_rank, ms = time_launches(torch, prob, stream, steps, warmup, dist, clocks)
    if world == 1:
        ms_one = ms
    agg = total_flops / (ms * 1e-3) / 1e12
    one = total_flops / (ms_one * 1e-3) / 1e12 if ms_one else None
    res = {"workload": cfg["desc"], "scaling": "strong", "experts": cfg["b"], "n_gpus": world,
           "tflops": round(agg, 2), "tflops_per_gpu": round(agg / world, 2), "ms_per_step": round(ms, 4),
           "steps": steps, "ranges": [list(gg.expert_shard(cfg["b"], world, r)) for r in range(world)],
           "tflops_1gpu_same_run": round(one, 2) if one else None,
           "efficiency_vs_1gpu": round(agg / (world * one), 4) if one else None,
           "rank0_clocks": clocks.summary(),
           "rank0_roofline": roofline(prob.flops, prob.alg_bytes, ms_rank, peaks, peak_src, load_traffic("E"),
                                      prob.backend.detail())}
    if allgather and dist:
        gathered = torch.empty(world * prob.rows, cfg["n"], device="cuda", dtype=prob.out.dtype)
        for _ in range(2):
            dist.all_gather_into_tensor(gathered, prob.out)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(5):
            dist.all_gather_into_tensor(gathered, prob.out)
        a1.record()
        a1.synchronize()
        res["allgather"] = {"ms": round(max_over_ranks(torch, dist, a0.elapsed_time(a1) / 5), 4),
                            "bytes_per_rank": prob.rows * cfg["n"] * 2, "how": "NCCL all_gather_into_tensor"}
        del gathered
    prob.release()
    del prob
    torch.cuda.empty_cache()
    return res


def e2e_leg(torch, gg, prob, stream, dist, steps):
    """End to end through the C ABI with host buffers: every step copies its x and w from pinned
    host memory and its output back. Two device buffer sets (each with its own prepared handle)
    let step i+1's host->device copies run on a copy stream while step i computes and copies
    back, as a serving loop would."""
    s = stream.cuda_stream
    x, w, out = prob.x, prob.w, prob.out
    cfg = prob.cfg
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    hw = torch.empty(w.shape, dtype=w.dtype, pin_memory=True)
    ho = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    hx.copy_(x)
    hw.copy_(w)
    sets = [(x, w, out, prob.backend)]
    x2, w2, out2 = torch.empty_like(x), torch.empty_like(w), torch.empty_like(out)
    b2 = gg.make_b200_backend()
    for key, val in prob.opts:
        b2.set_option(key, val)
    if b2.prepare(gg.DTYPES[cfg["dtype"]], prob.group_m, cfg["n"], cfg["k"], x2.data_ptr(), w2.data_ptr(),
                  out2.data_ptr(), s):
        raise SystemExit("prepare refused the second buffer set")
    sets.append((x2, w2, out2, b2))
    copy_stream = torch.cuda.Stream()
    copied = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    torch.cuda.synchronize()

    def e2e_step(i):
        xd, wd, od, be = sets[i % 2]
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(done[i % 2])  # the set's previous step has finished with it
            xd.copy_(hx, non_blocking=True)
            wd.copy_(hw, non_blocking=True)
            copied[i % 2].record(copy_stream)
        with torch.cuda.stream(stream):
            stream.wait_event(copied[i % 2])
            be.run(s)
            ho[i % 2].copy_(od, non_blocking=True)
            done[i % 2].record(stream)

    for i in range(2):  # warm-up of both sets
        e2e_step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(copy_stream)
    for i in range(steps):
        e2e_step(i)
    ev1.record(stream)
    ev1.synchronize()
    e2e_ms = ev0.elapsed_time(ev1) / steps
    for _, _, _, be in sets:
        if be.device_status(s) != 0:
            raise SystemExit("kernel reported a bounded-wait timeout in the end-to-end steps")
    b2.release()
    del x2, w2, out2
    return max_over_ranks(torch, dist, e2e_ms), int(hx.numel() * 2 + hw.numel() * 2), int(ho[0].numel() * 2)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="L", choices=sorted(CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--sustained-s", type=float, default=2.5,
                    help="seconds of the back-to-back sustained leg after the timed region (0 = skip)")
    ap.add_argument("--no-config-e", action="store_true", help="skip the config E strong-scaling leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allgather", action="store_true",
                    help="also time an NCCL all-gather of config E's sharded outputs")
    ap.add_argument("--variant", type=int, default=-1)
    ap.add_argument("--opt", action="append", default=[], metavar="KEY=VALUE",
                    help="gg_set_option knob for the headline problem's handle (repeatable), e.g. sched=0")
    ap.add_argument("--op", default="forward", choices=["forward", "dgrad", "wgrad"],
                    help="dgrad/wgrad: time a backward grouped GEMM on one GPU beside a per-expert "
                         "cuBLAS loop (not the headline line)")
    ap.add_argument("--vs-loop", action="store_true",
                    help="with --op forward: the same one-GPU comparison with a per-expert cuBLAS loop "
                         "in place of the headline line")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    if (args.op != "forward" or args.vs_loop) and args.impl == "ours":
        return run_vs_loop(args, cfg)

    if args.impl == "reference":
        return run_reference(args, cfg)

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    gg = load_package()
    peaks, peak_src = measured_peaks()
    total_groups, (g0, g1) = shard_of(cfg, world, rank, gg)
    stream = torch.cuda.Stream()
    opts = []
    for kv in args.opt:
        key, _, val = kv.partition("=")
        opts.append((key, int(val)))
    prob = Problem(gg, torch, cfg, g0, g1, 1000 + rank, stream, args.variant, opts)
    n, k = cfg["n"], cfg["k"]

    # ---- device-timed steps (inputs resident in HBM) ----
    clocks = ClockSampler(local_rank)
    ms_step_rank, ms_step = time_launches(torch, prob, stream, args.steps, args.warmup, dist, clocks)
    total_flops = 2.0 * sum(group_sizes(cfg, 0, total_groups)) * n * k
    value = total_flops / (ms_step * 1e-3) / 1e12
    detail = prob.backend.detail()
    roof = roofline(prob.flops, prob.alg_bytes, ms_step_rank, peaks, peak_src, load_traffic(args.config), detail)

    # ---- end to end through the C ABI with host buffers ----
    e2e_ms, h2d, d2h = e2e_leg(torch, gg, prob, stream, dist, max(1, min(args.e2e_steps, args.steps)))
    e2e = {"value": round(total_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
           "steps": max(1, min(args.e2e_steps, args.steps)),
           "path": "per step: pinned host x,w -> device, gg_run, out -> pinned host; two buffer sets so the "
                   "next step's copies overlap this step's GEMM"}

    # ---- config E sharded over the GPUs, strong scaling ----
    config_e = None
    if not args.no_config_e and args.config != "E":
        config_e = config_e_leg(torch, gg, dist, world, rank, local_rank, stream, min(args.steps, 20), args.warmup,
                                args.allgather, peaks, peak_src)

    # ---- sustained: seconds of back-to-back launches at the power cap (not in value); last, so
    # the power-capped state it ends in does not reach the other legs ----
    sustained = None
    if args.sustained_s > 0:
        sustained = sustained_leg(torch, prob, stream, dist, local_rank, args.sustained_s, peaks)
    prob.release()
    del prob
    torch.cuda.empty_cache()

    if dist:
        dist.barrier()
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return 0

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak"
        if cfg["per_gpu"] else "strong",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic N(0,1) (torch generator on the device), bf16; random expert weights",
        "config": {"workload": cfg["desc"], "global_batch": total_groups * cfg["m"], "experts": total_groups,
                   "parallelism": f"ep{world}", "l2": "inputs larger than L2 (no flush)",
                   "per_gpu_tflops": round(value / world, 2),
                   "pct_of_datasheet_dense_peak": round(100 * value / world / DATASHEET_TFLOPS, 2)},
        "roofline": roof,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "detail": detail,
    }
    if sustained:
        line["sustained"] = sustained
    if config_e:
        line["config_E"] = config_e
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
