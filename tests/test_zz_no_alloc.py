"""gg_run_noalloc: the entry point for callers that cannot allocate device memory.

Such callers (an engine whose memory pool already owns the GPU's memory, a plugin host with a
fixed budget, a path that must not call cudaMalloc because it can synchronise the device) get
the grouped GEMM with the library's scratch held in a fixed device array instead of allocated
buffers. These tests call it through the C ABI and check it against the regular
gg_prepare/gg_run path on calls in a row, with the reference's pass rule
|got - ref| <= 1e-2 + 1e-2 * |ref|. This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def _inputs(torch, orc, group_m, n, k, dtype):
    x, w = orc.make_inputs(group_m, n, k, dtype)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    return xd, wd


def _regular(gg, torch, group_m, n, k, dtype, xd, wd):
    out = torch.zeros(sum(group_m) * n, dtype=torch.int16, device="cuda")
    b = gg.B200Backend()
    s = torch.cuda.current_stream().cuda_stream
    assert b.prepare(dtype, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    assert b.device_status(s) == 0
    b.release()
    return out.cpu().numpy().view(np.uint16)


def _close(orc, got_bits, want_bits, dtype):
    got = orc.to_f32(got_bits, dtype)
    want = orc.to_f32(want_bits, dtype)
    return orc.check(got, want)


def _poisoned(torch, elems):
    return torch.full((elems,), 0x7E5A, dtype=torch.int16, device="cuda")


def test_noalloc_back_to_back_calls_match_regular_path(gg, orc):
    """Two different problems queued back to back on one stream without waiting (the second call
    overwrites the shared offsets while the first may still be queued), then a waited call whose
    status covers all three kernels; every output is checked."""
    torch = _torch()
    s = torch.cuda.current_stream().cuda_stream
    cases = [
        ([256] * 4, 512, 384, gg.BF16),                   # BASELINE config T
        ([0, 130, 1, 300, 77], 264, 200, gg.FP16),        # empty/ragged groups, K and N tails
    ]
    prepared = []
    for group_m, n, k, dtype in cases:
        xd, wd = _inputs(torch, orc, group_m, n, k, dtype)
        want = _regular(gg, torch, group_m, n, k, dtype, xd, wd)
        prepared.append((group_m, n, k, dtype, xd, wd, _poisoned(torch, sum(group_m) * n), want))
    torch.cuda.synchronize()
    for group_m, n, k, dtype, xd, wd, out, _ in prepared:
        rc, why, st = gg.run_noalloc(dtype, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s)
        assert rc == gg.GG_OK and st == 0, (rc, why, st)
    group_m, n, k, dtype, xd, wd, _, want0 = prepared[0]
    again = _poisoned(torch, sum(group_m) * n)
    rc, why, st = gg.run_noalloc(dtype, group_m, n, k, xd.data_ptr(), wd.data_ptr(), again.data_ptr(), s,
                                 wait=True)
    assert rc == gg.GG_OK and st == 0, (rc, why, hex(st))
    torch.cuda.synchronize()
    outputs = [(p[6], p[7], p[3], p[0]) for p in prepared] + [(again, want0, dtype, group_m)]
    for out, want, dt, gm in outputs:
        bad, mx = _close(orc, out.cpu().numpy().view(np.uint16), want, dt)
        assert bad == 0, (gm, bad, mx)


def test_noalloc_repeated_call_without_waiting(gg, orc):
    torch = _torch()
    s = torch.cuda.current_stream().cuda_stream
    group_m, n, k = [1000] * 3, 2880, 2880
    xd, wd = _inputs(torch, orc, group_m, n, k, gg.BF16)
    want = _regular(gg, torch, group_m, n, k, gg.BF16, xd, wd)
    outs = [_poisoned(torch, sum(group_m) * n) for _ in range(2)]
    for i, out in enumerate(outs):
        rc, why, st = gg.run_noalloc(gg.BF16, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s,
                                     wait=i == len(outs) - 1)
        assert rc == gg.GG_OK and st == 0, (rc, why, hex(st))
    torch.cuda.synchronize()
    for out in outs:
        bad, mx = _close(orc, out.cpu().numpy().view(np.uint16), want, gg.BF16)
        assert bad == 0, (bad, mx)


def test_noalloc_refuses_more_groups_than_its_scratch_holds(gg):
    torch = _torch()
    t = torch.zeros(64, dtype=torch.int16, device="cuda")
    rc, why, _ = gg.run_noalloc(gg.BF16, [1] * 1025, 8, 8, t.data_ptr(), t.data_ptr(), t.data_ptr())
    assert rc == gg.GG_NOT_SUPPORTED and "1024" in why
