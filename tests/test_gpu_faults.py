"""Failure detection on the GPU without faulting it.

Every wait in the kernel is bounded. The test hook "test_stall" makes the pair leader skip the
loads of cluster 0's first pipeline stage, so the MMA thread's wait on that stage never
completes: after timeout_ms it records a status code (0x1000 | role << 8 | barrier), every role
of every CTA leaves its loop, Tensor Memory is freed and the kernel returns. The host reads the
status with gg_device_status, and the same context must then compute correctly. The reference
has no counterpart (its kernel can only trap, ck_kernel/fast_epilogue.hpp:38-41).
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROLE_MMA = 2 << 8
ROLE_EPILOGUE = 3 << 8


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


@pytest.mark.parametrize("variant", [0, 1])
def test_stalled_wait_reports_status_and_context_survives(gg, orc, variant):
    torch = _torch()
    group_m, n, k = [256, 256], 512, 256
    x, w = orc.make_inputs(group_m, n, k, gg.BF16)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    out = torch.zeros(sum(group_m) * n, dtype=torch.int16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    b = gg.B200Backend()
    b.set_option("variant", variant)
    b.set_option("timeout_ms", 200)
    b.set_option("test_stall", 1)
    assert b.prepare(gg.BF16, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    t0 = time.time()
    b.run(s)
    st = b.device_status(s)
    elapsed = time.time() - t0
    assert st & 0x1000, hex(st)
    # the MMA thread (waiting on stage 0) or the epilogue (waiting on accumulator 0) runs out first
    assert (st & 0xF00) in (ROLE_MMA, ROLE_EPILOGUE) and (st & 0xFF) == 0, hex(st)
    assert elapsed < 30
    assert b.device_status(s) == 0  # reading clears it

    # the context is still usable: a normal run is correct
    ok = gg.B200Backend()
    ok.set_option("variant", variant)
    assert ok.prepare(gg.BF16, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    ok.run(s)
    assert ok.device_status(s) == 0
    got = out.cpu().numpy().view(np.uint16)
    assert orc.check16(got, orc.grouped_gemm_f32(x, w, group_m, gg.BF16), gg.BF16)[0] == 0


def test_aborted_split_k_launch_is_cleaned_up(gg, orc):
    """A split-K launch that times out leaves arrival counters behind; gg_device_status clears
    them, so the next launch of the same prepared problem is correct."""
    torch = _torch()
    group_m, n, k = [512], 1024, 2048
    x, w = orc.make_inputs(group_m, n, k, gg.BF16)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    out = torch.zeros(sum(group_m) * n, dtype=torch.int16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    b = gg.B200Backend()
    b.set_option("variant", 0)
    b.set_option("split", 2)
    b.set_option("timeout_ms", 200)
    b.set_option("test_stall", 1)
    assert b.prepare(gg.BF16, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    assert b.device_status(s) & 0x1000
    b.set_option("test_stall", 0)
    assert b.prepare(gg.BF16, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    assert b.device_status(s) == 0
    got = out.cpu().numpy().view(np.uint16)
    assert orc.check16(got, orc.grouped_gemm_f32(x, w, group_m, gg.BF16), gg.BF16)[0] == 0
