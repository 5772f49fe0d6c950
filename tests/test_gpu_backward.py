"""GPU parity of the backward grouped GEMMs (dgrad, wgrad) against the CPU oracle, through the
C ABI (gg_prepare_grad + gg_run).

    dgrad: dx[rows of g] = dy[rows of g] @ w[g]          dx [sum(M), K]
    wgrad: dw[g] = dy[rows of g]^T @ x[rows of g]        dw [G, N, K], zero for an empty expert

The reference's vendored Primus-Turbo grouped GEMM defines both calls
(third_party/primus_turbo/kernels/hipblaslt_grouped_gemm.cu:80-96,199-240). Tolerance is the
reference's pass rule (bench/bench_main.cpp:264-270): |got - ref| <= 1e-2 + 1e-2 * |ref|, NaN
fails, over the full output. Outputs start as a canary pattern, so a missed store fails, and a
guard region after the output must stay untouched.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = 0x7E5A
GUARD = 4096


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def upload(torch, bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()


def run_grad(gg, op, group_m, n, k, dtype, dy, x, w, variant=-1, bn=0, split=0, band=0, runs=1, opts=None):
    """Prepare and run one backward op; returns (output bits, detail)."""
    torch = _torch()
    total = int(sum(group_m))
    rows = total if op == gg.OP_DGRAD else len(group_m) * n
    out = torch.full((rows * k + GUARD,), CANARY, dtype=torch.int16, device="cuda")
    b = gg.B200Backend()
    if variant >= 0:
        b.set_option("variant", variant)
    if bn:
        b.set_option("bn", bn)
    if split:
        b.set_option("split", split)
    if band:
        b.set_option("band", band)
    for key, val in (opts or {}).items():
        b.set_option(key, val)
    s = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: t.data_ptr() if t is not None and t.numel() else 0  # noqa: E731
    if op == gg.OP_DGRAD:
        why = b.prepare_grad(op, dtype, group_m, n, k, dy_ptr=ptr(dy), w_ptr=ptr(w), dx_ptr=out.data_ptr(), stream=s)
    else:
        why = b.prepare_grad(op, dtype, group_m, n, k, dy_ptr=ptr(dy), x_ptr=ptr(x), dw_ptr=out.data_ptr(), stream=s)
    assert why == "", why
    for _ in range(runs):
        b.run(s)
    torch.cuda.synchronize()
    assert b.device_status(s) == 0
    res = out.cpu().numpy().view(np.uint16)
    assert np.all(res[rows * k:] == CANARY), "store past the end of the output"
    detail = b.detail()
    b.release()
    return res[:rows * k].reshape(rows, k), detail


def grad_case(gg, orc, op, group_m, n, k, dtype, variants=(-1,), **kw):
    torch = _torch()
    dy, x, w = orc.make_grad_inputs(group_m, n, k, dtype)
    if op == gg.OP_DGRAD:
        ref = orc.grouped_dgrad_f32(dy, w, group_m, dtype)
    else:
        ref = orc.grouped_wgrad_f32(dy, x, group_m, dtype).reshape(-1, k)
    dyd, xd, wd = upload(torch, dy), upload(torch, x), upload(torch, w)
    for v in variants:
        got, detail = run_grad(gg, op, group_m, n, k, dtype, dyd, xd, wd, variant=v, **kw)
        assert ("dgrad" if op == gg.OP_DGRAD else "wgrad") in detail, detail
        bad, mx, first = orc.check16(got, ref, dtype)
        assert bad == 0, f"variant {v} ({detail}): {bad} mismatches, first at {divmod(first, k)}, max abs {mx}"


ALL_VARIANTS = (0, 1, 2)
OPS = ("dgrad", "wgrad")


def _op(gg, name):
    return gg.OP_DGRAD if name == "dgrad" else gg.OP_WGRAD


@pytest.mark.parametrize("name", OPS)
@pytest.mark.parametrize("dtype", [0, 1])
def test_tiny_all_variants(gg, orc, name, dtype):
    # the shape of BASELINE config T (B=4, M=256, N=512, K=384)
    grad_case(gg, orc, _op(gg, name), [256] * 4, 512, 384, dtype, ALL_VARIANTS)


@pytest.mark.parametrize("name", OPS)
@pytest.mark.parametrize("dtype", [0, 1])
def test_unbalanced_empty_groups_and_tails(gg, orc, name, dtype):
    # empty experts, groups shorter than a tile and than a 64-token atom, N and K tails
    group_m = [0, 1, 127, 128, 129, 0, 300, 5, 0, 257]
    grad_case(gg, orc, _op(gg, name), group_m, 264, 200, dtype, ALL_VARIANTS)


@pytest.mark.parametrize("name", OPS)
def test_padded_shape(gg, orc, name):
    # shapes/pad_test.csv 9003: B=2, M=300, N=1000, K=2048 (fp16)
    grad_case(gg, orc, _op(gg, name), [300] * 2, 1000, 2048, 1, ALL_VARIANTS)


@pytest.mark.parametrize("name", OPS)
@pytest.mark.parametrize("variant,bn", [(0, 128), (1, 192), (1, 128), (1, 64), (2, 64)])
def test_tile_widths(gg, orc, name, variant, bn):
    grad_case(gg, orc, _op(gg, name), [300, 0, 17, 513], 320, 1000, 0, (variant,), bn=bn)


@pytest.mark.parametrize("variant,split", [(0, 2), (1, 3), (2, 4)])
def test_dgrad_split_k(gg, orc, variant, split):
    # split-K over N (the dgrad reduction); two launches in a row reuse the arrival counters
    grad_case(gg, orc, gg.OP_DGRAD, [300, 0, 17, 513], 1000, 256, 0, (variant,), split=split, runs=2)


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("group_m,n,k,variant,bn,mode", [
    ([300, 0, 65, 1000, 7], 512, 384, 0, 256, 3),     # both operands in chunk boxes, pair tile
    ([300, 0, 65, 1000, 7], 320, 448, 0, 128, 3),     # N tail inside a 256-row tile, one chunk of x per CTA
    ([130, 64, 1], 448, 200, 1, 192, 1),              # K % 64 != 0: dy in chunk boxes, x in 2-D boxes
    ([130, 64, 1], 200, 256, 1, 256, 2),              # N % 64 != 0: x in chunk boxes (4 per box)
    ([500, 33], 256, 320, 2, 128, 3),                 # one-CTA 128 x 128 tile
    ([2000, 129, 0, 64], 768, 1024, -1, 0, 3),        # automatic tiling
])
def test_wgrad_chunk_boxes_match_2d_boxes(gg, orc, dtype, group_m, n, k, variant, bn, mode):
    """wgrad's MN-major operands loaded through the 3-D chunk view (one box per operand and atom)
    give the same bits as one 2-D box per 64-column chunk, and pass the oracle's full compare;
    shapes whose N (dy) or K (x) is not a multiple of 64 keep the 2-D boxes for that operand."""
    torch = _torch()
    dy, x, w = orc.make_grad_inputs(group_m, n, k, dtype)
    ref = orc.grouped_wgrad_f32(dy, x, group_m, dtype).reshape(-1, k)
    dyd, xd, wd = upload(torch, dy), upload(torch, x), upload(torch, w)
    got = {}
    for chunks in (0, 1):
        res, detail = run_grad(gg, gg.OP_WGRAD, group_m, n, k, dtype, dyd, xd, wd, variant=variant, bn=bn, runs=2,
                               opts={"tma_chunks": chunks})
        tag = {3: "chunk-boxes ", 1: "chunk-boxes(dy)", 2: "chunk-boxes(x)"}[mode]
        assert (tag in detail + " ") == (chunks == 1), detail
        bad, mx, first = orc.check16(res, ref, dtype)
        assert bad == 0, f"tma_chunks={chunks} ({detail}): {bad} mismatches, first at {divmod(first, k)}, max abs {mx}"
        got[chunks] = res
    assert np.array_equal(got[0], got[1])


def test_wgrad_every_expert_empty_writes_zeros(gg, orc):
    torch = _torch()
    group_m, n, k = [0, 0, 0], 136, 72
    got, detail = run_grad(gg, gg.OP_WGRAD, group_m, n, k, 0, None, None, None)
    assert np.all(got == 0), detail


def test_wgrad_long_reduction(gg, orc):
    # few output tiles, thousands of tokens per expert: a long K loop per tile
    grad_case(gg, orc, gg.OP_WGRAD, [4096, 1500], 256, 256, 0, ALL_VARIANTS)


def test_backward_refusals(gg):
    torch = _torch()
    buf = torch.zeros(1 << 16, dtype=torch.int16, device="cuda")
    p = buf.data_ptr()
    b = gg.B200Backend()
    b.set_option("bn", 96)  # 96 columns per CTA is not a whole number of 64-wide boxes
    b.set_option("variant", 1)
    assert "multiple of 64" in b.prepare_grad(gg.OP_DGRAD, 0, [8], 64, 64, dy_ptr=p, w_ptr=p, dx_ptr=p)
    b = gg.B200Backend()
    b.set_option("split", 2)
    assert "wgrad" in b.prepare_grad(gg.OP_WGRAD, 0, [8], 64, 64, dy_ptr=p, x_ptr=p, dw_ptr=p)


def test_forward_after_backward_on_one_handle(gg, orc):
    """A handle prepared for wgrad (per-group tensor maps) and then for the forward op computes
    the forward op correctly."""
    torch = _torch()
    group_m, n, k = [100, 0, 200], 256, 128
    dy, x, w = orc.make_grad_inputs(group_m, n, k, 0)
    dyd, xd, wd = upload(torch, dy), upload(torch, x), upload(torch, w)
    dw = torch.zeros(len(group_m) * n * k, dtype=torch.int16, device="cuda")
    out = torch.zeros(sum(group_m) * n, dtype=torch.int16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    b = gg.B200Backend()
    assert b.prepare_grad(gg.OP_WGRAD, 0, group_m, n, k, dy_ptr=dyd.data_ptr(), x_ptr=xd.data_ptr(),
                          dw_ptr=dw.data_ptr(), stream=s) == ""
    b.run(s)
    assert b.prepare(0, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    assert b.device_status(s) == 0
    ref_dw = orc.grouped_wgrad_f32(dy, x, group_m, 0).reshape(-1, k)
    assert orc.check16(dw.cpu().numpy().view(np.uint16).reshape(-1, k), ref_dw, 0)[0] == 0
    ref = orc.grouped_gemm_f32(x, w, group_m, 0)
    assert orc.check16(out.cpu().numpy().view(np.uint16).reshape(-1, n), ref, 0)[0] == 0


@pytest.mark.parametrize("name", OPS)
def test_config_l_size_two_experts_vs_torch_fp32(gg, name):
    """BASELINE config L's shape (B=8, M=4096, N=4096, K=7168, bf16): the whole output of the
    first and the last expert against a torch fp32 matmul of the same bf16 inputs."""
    torch = _torch()
    B, M, N, K = 8, 4096, 4096, 7168
    gen = torch.Generator(device="cuda").manual_seed(11)
    dy = torch.randn(B * M, N, device="cuda", generator=gen).to(torch.bfloat16)
    group_m = [M] * B
    s = torch.cuda.current_stream().cuda_stream
    b = gg.B200Backend()
    if name == "dgrad":
        w = torch.randn(B, N, K, device="cuda", generator=gen).to(torch.bfloat16)
        dx = torch.empty(B * M, K, device="cuda", dtype=torch.bfloat16)
        assert b.prepare_grad(gg.OP_DGRAD, gg.BF16, group_m, N, K, dy_ptr=dy.data_ptr(), w_ptr=w.data_ptr(),
                              dx_ptr=dx.data_ptr(), stream=s) == ""
    else:
        x = torch.randn(B * M, K, device="cuda", generator=gen).to(torch.bfloat16)
        dw = torch.empty(B, N, K, device="cuda", dtype=torch.bfloat16)
        assert b.prepare_grad(gg.OP_WGRAD, gg.BF16, group_m, N, K, dy_ptr=dy.data_ptr(), x_ptr=x.data_ptr(),
                              dw_ptr=dw.data_ptr(), stream=s) == ""
    b.run(s)
    assert b.device_status(s) == 0
    for g in (0, B - 1):
        rows = slice(g * M, (g + 1) * M)
        if name == "dgrad":
            ref = dy[rows].float() @ w[g].float()
            got = dx[rows].float()
        else:
            ref = dy[rows].float().t() @ x[rows].float()
            got = dw[g].float()
        bad = ((got - ref).abs() > 1e-2 + 1e-2 * ref.abs()) | torch.isnan(got)
        assert int(bad.sum()) == 0, (name, g, int(bad.sum()), float((got - ref).abs().max()))
    b.release()


@pytest.mark.parametrize("args", [["--op", "forward", "--vs-loop"], ["--op", "dgrad"], ["--op", "wgrad"]])
def test_bench_vs_loop_leg(args):
    """bench.py's one-GPU comparison leg (each op beside a per-expert cuBLAS loop, the two arms
    alternating in rounds) on config T: one JSON line whose output agrees with cuBLAS everywhere."""
    import json
    import os
    import subprocess
    import sys

    _torch()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--config", "T", "--steps", "10",
                        "--warmup", "3", *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["op"] == args[1] and line["rounds"] == 5 and line["gpu_launches"] == 10
    assert line["check_vs_cublas"]["outside_tolerance"] == 0
    assert line["value"] > 0 and line["cublas_loop"]["value"] > 0 and line["ratio_vs_loop"] > 0
    assert len(line["rounds_tflops"]["ours"]) == len(line["rounds_tflops"]["loop"]) == 5
