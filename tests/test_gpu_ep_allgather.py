"""Expert parallelism on two or more GPUs: each rank runs the kernel on its contiguous expert
shard (no collective on the GEMM path), then the optional NCCL all-gather of the outputs (the one
bench.py --allgather times) assembles them. The gathered output must equal the unsharded run on
one GPU bit for bit and pass the reference's check against the CPU oracle. Skipped on a box with
fewer than two GPUs; the same host logic runs on CPU ranks in tests/test_ep_shard.py."""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_sharded_outputs_all_gather_to_the_unsharded_result(tmp_path):
    import torch

    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs two GPUs")
    world = min(n, 4)
    out = tmp_path / "res.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "ep_allgather_worker.py"), str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-6000:])
    res = json.loads(out.read_text())
    assert res["world"] == world
    assert res["bitwise_equal_to_unsharded"], res
    assert res["oracle_mismatches"] == 0, res
