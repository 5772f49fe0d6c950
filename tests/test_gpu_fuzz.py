"""Seeded random cases over the scheduling options, all three operations, checked in full
against the CPU oracle (the reference's pass rule, bench/bench_main.cpp:264-270).

Each case draws ragged group sizes (some empty), N and K with tails, a dtype, and a random mix
of the options that change the kernel's schedule: variant, tile width, split count and form
(every tile or only the last partial wave) or stream-K kind, raster order and band, a capped
grid (so small problems still have several waves), and static or dynamic tile dispatch. A combination the library refuses must be
refused with one of its documented reasons; every accepted one must match the oracle within
tolerance, give the same bits on a second run, and leave the guard region after the output
untouched.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0x7E5A
GUARD = 2048
REFUSALS = ("multiple of 64", "split exceeds", "split_tail=1", "split-K is not available", "no kernel variant",
            "wider than the variant", "stream_k: this tiling", "stream-K is not available")


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def draw_case(rng):
    G = int(rng.integers(1, 9))
    group_m = [int(v) if rng.random() > 0.2 else 0 for v in rng.integers(1, 700, size=G)]
    n = 8 * int(rng.integers(1, 120))
    k = 8 * int(rng.integers(1, 150))
    op = ("forward", "dgrad", "wgrad")[int(rng.integers(0, 3))]
    dtype = int(rng.integers(0, 2))
    opts = {}
    if rng.random() < 0.6:
        opts["variant"] = int(rng.integers(0, 3))
    if rng.random() < 0.4:
        opts["bn"] = 32 * int(rng.integers(1, 9))
    if rng.random() < 0.5:
        opts["split"] = int(rng.integers(1, 5))
        opts["split_tail"] = int(rng.integers(-1, 2))
    if rng.random() < 0.3:
        opts["raster"] = int(rng.integers(0, 2))
        opts["band"] = int(rng.integers(1, 9))
    if rng.random() < 0.5:
        opts["max_ctas"] = int(rng.choice([4, 6, 10, 22]))
    if rng.random() < 0.5:
        opts["sched"] = int(rng.integers(0, 2))  # static or dynamic tile dispatch (else automatic)
    if rng.random() < 0.3:
        opts["half_tiles"] = int(rng.integers(0, 2))
    if rng.random() < 0.5:
        opts["tail_launch"] = int(rng.integers(0, 2))  # otherwise automatic (skewed remainders)
    if rng.random() < 0.4:
        opts["tile_order"] = int(rng.integers(0, 2))  # wgrad: group order or interleaved (else automatic)
    if rng.random() < 0.3:
        opts["tma_chunks"] = 0  # wgrad: one 2-D box per 64-column chunk instead of the 3-D chunk view
    return group_m, n, k, op, dtype, opts


def draw_case_stream_k(rng):
    """A case as above with stream-K (automatic, off, or forced to either kind) in place of
    split-K, tile widths in steps of 16, and a capped grid more often."""
    group_m, n, k, op, dtype, opts = draw_case(rng)
    opts.pop("split", None)
    opts.pop("split_tail", None)
    if rng.random() < 0.7:
        opts["bn"] = 16 * int(rng.integers(1, 17))
    opts["stream_k"] = int(rng.integers(-1, 3))
    if rng.random() < 0.7:
        opts["max_ctas"] = int(rng.choice([4, 6, 10, 22, 40]))
    return group_m, n, k, op, dtype, opts


@pytest.mark.parametrize("seed", range(96))
def test_random_case(gg, orc, seed):
    check_case(gg, orc, draw_case(np.random.default_rng(1000 + seed)))


@pytest.mark.parametrize("seed", range(48))
def test_random_case_stream_k(gg, orc, seed):
    check_case(gg, orc, draw_case_stream_k(np.random.default_rng(5000 + seed)))


def check_case(gg, orc, drawn):
    torch = _torch()
    group_m, n, k, op, dtype, opts = drawn
    total = sum(group_m)
    s = torch.cuda.current_stream().cuda_stream
    b = gg.B200Backend()
    for key, val in opts.items():
        b.set_option(key, val)
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()  # noqa: E731
    if op == "forward":
        x, w = orc.make_inputs(group_m, n, k, dtype)
        rows, cols = total, n
        out = torch.full((rows * cols + GUARD,), CANARY, dtype=torch.int16, device="cuda")
        xd, wd = up(x), up(w)
        why = b.prepare(dtype, group_m, n, k, xd.data_ptr() if total else 0, wd.data_ptr(), out.data_ptr(), s)
        ref = orc.grouped_gemm_f32(x, w, group_m, dtype) if not why else None
    else:
        dy, x, w = orc.make_grad_inputs(group_m, n, k, dtype)
        dyd, xd, wd = up(dy), up(x), up(w)
        ptr = lambda t: t.data_ptr() if t.numel() else 0  # noqa: E731
        if op == "dgrad":
            rows, cols = total, k
            out = torch.full((rows * cols + GUARD,), CANARY, dtype=torch.int16, device="cuda")
            why = b.prepare_grad(gg.OP_DGRAD, dtype, group_m, n, k, dy_ptr=ptr(dyd), w_ptr=ptr(wd),
                                 dx_ptr=out.data_ptr(), stream=s)
            ref = orc.grouped_dgrad_f32(dy, w, group_m, dtype) if not why else None
        else:
            rows, cols = len(group_m) * n, k
            out = torch.full((rows * cols + GUARD,), CANARY, dtype=torch.int16, device="cuda")
            why = b.prepare_grad(gg.OP_WGRAD, dtype, group_m, n, k, dy_ptr=ptr(dyd), x_ptr=ptr(xd),
                                 dw_ptr=out.data_ptr(), stream=s)
            ref = orc.grouped_wgrad_f32(dy, x, group_m, dtype).reshape(-1, k) if not why else None
    case = (op, group_m, n, k, dtype, opts)
    if why:
        assert any(r in why for r in REFUSALS), (case, why)
        return
    first_res = None
    for _ in range(2):  # twice: split-K arrival counters must be back at zero
        b.run(s)
        assert b.device_status(s) == 0, (case, b.detail())
        res = out.cpu().numpy().view(np.uint16)
        if first_res is None:
            first_res = res.copy()
        else:  # the same bits again: the partial sums are added in a fixed order
            assert np.array_equal(first_res, res), (case, b.detail(), "second run differs")
        assert np.all(res[rows * cols:] == CANARY), (case, b.detail(), "store past the end")
        if rows:
            bad, mx, first = orc.check16(res[:rows * cols].reshape(rows, cols), ref, dtype)
            assert bad == 0, (case, b.detail(), bad, mx, first)
