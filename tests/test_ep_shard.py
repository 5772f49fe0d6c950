"""Expert-parallel sharding on CPU ranks (gloo, world size 2), no GPU.

The multi-GPU path shards experts contiguously (gg_expert_shard) and runs the single-GPU kernel
on each rank's experts; the GEMM path has no collective. These tests run that host logic with
the CPU oracle standing in for the kernel: every rank computes its experts' rows, an all-gather
assembles them, and the result must equal the single-process computation bit for bit (each
output element depends only on its own row and expert).
"""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, load_oracle, load_package


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


GROUP_M = [7, 0, 33, 16, 5, 64, 1]  # unbalanced, one empty expert
N, K, DT = 40, 72, 0


def _rank_main(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    gg = load_package()
    orc = load_oracle()
    g0, g1 = gg.expert_shard(len(GROUP_M), world, rank)
    x, w = orc.make_inputs(GROUP_M, N, K, DT)
    row_off = np.concatenate([[0], np.cumsum(GROUP_M)])
    r0, r1 = int(row_off[g0]), int(row_off[g1])
    # the rank's shard: its experts' rows of x and its slice of w, like bench.py's per-rank inputs
    local = orc.grouped_gemm_f32(np.ascontiguousarray(x[r0:r1]), np.ascontiguousarray(w[g0:g1]),
                                 GROUP_M[g0:g1], DT)
    # all-gather of variable-size row blocks: pad to the largest shard
    rows = torch.tensor([r1 - r0])
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, rows)
    cap = int(max(s.item() for s in sizes))
    buf = torch.zeros(cap, N)
    buf[: r1 - r0] = torch.from_numpy(local)
    parts = [torch.zeros(cap, N) for _ in range(world)]
    dist.all_gather(parts, buf)
    if rank == 0:
        full = np.concatenate([p[: int(s.item())].numpy() for p, s in zip(parts, sizes)])
        want = orc.grouped_gemm_f32(x, w, GROUP_M, DT)
        with open(result_path, "w") as f:
            json.dump({"equal": bool(np.array_equal(full, want)), "shape": list(full.shape)}, f)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_expert_shards_reassemble_exactly(gg, orc, tmp_path):
    out = tmp_path / "result.json"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(out)), nprocs=2, join=True, start_method="spawn")
    res = json.loads(out.read_text())
    assert res["equal"] and res["shape"] == [sum(GROUP_M), N]


def test_bench_shard_ranges_cover_the_job(gg):
    sys.path.insert(0, ROOT)
    try:
        import bench
    finally:
        sys.path.pop(0)
    for world in (1, 2, 4, 8):
        for name in ("L", "E"):
            cfg = bench.CONFIGS[name]
            seen = []
            for r in range(world):
                total, (g0, g1) = bench.shard_of(cfg, world, r, gg)
                seen.extend(range(g0, g1))
            assert seen == list(range(total))
            # weak scaling for L (8 experts per GPU), strong for E (256 in total)
            assert total == (8 * world if name == "L" else 256)


def test_reference_arm_prints_contract_line():
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "T",
                        "--steps", "2", "--warmup", "3"], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "impl", "cpu_baseline", "e2e", "higher_is_better", "config"):
        assert key in line
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
