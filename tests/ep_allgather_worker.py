"""Worker of tests/test_gpu_ep_allgather.py, one process per GPU under torchrun.

Each rank runs the B200 kernel (through the C ABI) on its contiguous expert shard of a small
config-E-like problem, then an NCCL all_gather_into_tensor assembles the shards' outputs, the
collective bench.py --allgather times. Rank 0 also runs the unsharded problem on its GPU and
writes, as JSON to argv[1], whether the gathered output equals it bit for bit and how it
compares with the CPU oracle under the reference's pass rule.
"""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from conftest import load_oracle, load_package  # noqa: E402

B, M, N, K, DT = 16, 192, 512, 640, 0  # balanced experts, as bench.py's config E


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    gg, orc = load_package(), load_oracle()
    group_m = [M] * B
    x, w = orc.make_inputs(group_m, N, K, DT)
    g0, g1 = gg.expert_shard(B, world, rank)
    xd = torch.from_numpy(x[g0 * M:g1 * M].view(np.int16)).cuda()
    wd = torch.from_numpy(np.ascontiguousarray(w[g0:g1]).view(np.int16)).cuda()
    out = torch.zeros((g1 - g0) * M, N, dtype=torch.int16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    be = gg.make_b200_backend()
    assert be.prepare(DT, group_m[g0:g1], N, K, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    be.run(s)
    assert be.device_status(s) == 0
    gathered = torch.empty(B * M, N, dtype=torch.int16, device="cuda")
    # NCCL has no 16-bit integer type: move the raw bits as bf16 (a bit-preserving view)
    dist.all_gather_into_tensor(gathered.view(torch.bfloat16), out.view(torch.bfloat16))
    torch.cuda.synchronize()
    if rank == 0:
        whole = torch.zeros(B * M, N, dtype=torch.int16, device="cuda")
        xa = torch.from_numpy(x.view(np.int16)).cuda()
        wa = torch.from_numpy(w.view(np.int16)).cuda()
        b2 = gg.make_b200_backend()
        assert b2.prepare(DT, group_m, N, K, xa.data_ptr(), wa.data_ptr(), whole.data_ptr(), s) == ""
        b2.run(s)
        assert b2.device_status(s) == 0
        torch.cuda.synchronize()
        g = gathered.cpu().numpy().view(np.uint16)
        bad, mx, _ = orc.check16(g, orc.grouped_gemm_f32(x, w, group_m, DT), DT)
        res = {"world": world, "bitwise_equal_to_unsharded": bool(torch.equal(gathered, whole)),
               "oracle_mismatches": bad, "max_abs": mx,
               "ranges": [list(gg.expert_shard(B, world, r)) for r in range(world)]}
        with open(out_path, "w") as f:
            json.dump(res, f)
        b2.release()
    be.release()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
