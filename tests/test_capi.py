"""CPU tests of the C ABI (no kernel launches): symbols, host-side argument checks, expert
sharding arithmetic and option handling. Mirrors the reference's N/A behaviour for shapes a
backend refuses (bench/bench_main.cpp:469-472)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "gg_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gg_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(gg):
    lib = gg.load_library()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in gg.SIGNATURES, f"{n} has no ctypes signature"


def test_debug_library_exports_the_same_symbols(gg):
    """The bounds-checked debug build (-DGG_DEBUG) is the same C ABI."""
    path = os.path.join(os.path.dirname(gg.LIB_PATH), "libgg_b200_debug.so")
    assert os.path.exists(path), "build it with groupgemm-cktile-optimized_b200/build.py"
    lib = ctypes.CDLL(path)
    for n in declared_functions():
        assert hasattr(lib, n), n


def test_abi_version_and_name(gg):
    lib = gg.load_library()
    assert lib.gg_abi_version() == 1
    b = gg.B200Backend()
    assert b.name() == "b200"
    assert b.detail() == ""


@pytest.mark.parametrize("g,world", [(256, 8), (256, 1), (7, 3), (3, 8), (0, 2), (33, 4)])
def test_expert_shard_partitions_contiguously(gg, g, world):
    ranges = [gg.expert_shard(g, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == g
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_expert_shard_rejects_bad_args(gg):
    with pytest.raises(gg.GGError):
        gg.expert_shard(8, 0, 0)
    with pytest.raises(gg.GGError):
        gg.expert_shard(8, 2, 2)


def test_set_option(gg):
    b = gg.B200Backend()
    b.set_option("variant", 1)
    b.set_option("band", 4)
    b.set_option("timeout_ms", 500)
    b.set_option("max_ctas", 64)
    b.set_option("test_stall", 0)
    b.set_option("bn", 192)
    b.set_option("bn", 0)
    b.set_option("split", 2)
    b.set_option("split", 0)
    for key, val in (("split_tail", -1), ("split_tail", 0), ("split_tail", 1), ("raster", 1), ("raster", -1),
                     ("pdl", 0), ("pdl", 1), ("store", -1), ("store", 0), ("store", 1), ("stream_k", -1),
                     ("stream_k", 0), ("stream_k", 1), ("stream_k", 2), ("bn", 240), ("bn", 16), ("bn", 0),
                     ("sched", -1), ("sched", 0), ("sched", 1), ("half_tiles", -1), ("half_tiles", 0), ("half_tiles", 1),
                     ("tail_launch", -1), ("tail_launch", 0), ("tail_launch", 1), ("test_bounds", 0), ("test_bounds", 1),
                     ("tile_order", -1), ("tile_order", 0), ("tile_order", 1), ("tma_chunks", 0), ("tma_chunks", 1),
                     ("l2_a", -1), ("l2_a", 0), ("l2_a", 2), ("l2_b", 0), ("l2_b", 1), ("l2_b", 2)):
        b.set_option(key, val)
    for key, val in (("variant", 7), ("band", -1), ("timeout_ms", 0), ("test_stall", 2), ("bn", 100), ("bn", 288), ("split", 9),
                     ("split_tail", 2), ("raster", 2), ("pdl", 3), ("store", 2), ("bogus", 1), ("bn", 24), ("bn", 8),
                     ("stream_k", 3), ("stream_k", -2), ("sched", 2), ("sched", -2), ("half_tiles", 2), ("tail_launch", 2), ("test_bounds", 2),
                     ("tile_order", 2), ("tile_order", -2), ("tma_chunks", 2), ("tma_chunks", -1), ("l2_a", 3), ("l2_a", -2),
                     ("l2_b", -1), ("l2_b", 3)):
        with pytest.raises(gg.GGError):
            b.set_option(key, val)


ALIGNED = 0x10000


@pytest.mark.parametrize(
    "kw,reason",
    [
        (dict(dtype=5), "dtype"),
        (dict(group_m=[]), "group_num"),
        (dict(group_m=[4, -1]), "group_m"),
        (dict(k=100), "k must be a multiple of 8"),
        (dict(n=1000 + 4), "n must be a multiple of 8"),
        (dict(n=0), "n and k"),
        (dict(x=ALIGNED + 8), "16-byte aligned"),
        (dict(out=0), "non-null"),
        (dict(group_m=[1 << 30, 1 << 30]), "2^31"),
    ],
)
def test_prepare_refuses_unsupported_shapes(gg, kw, reason):
    args = dict(dtype=gg.BF16, group_m=[4, 4], n=64, k=64, x=ALIGNED, w=ALIGNED, out=ALIGNED)
    args.update(kw)
    b = gg.B200Backend()
    why = b.prepare(args["dtype"], args["group_m"], args["n"], args["k"], args["x"], args["w"], args["out"])
    assert reason in why
    with pytest.raises(gg.GGError):
        b.run()  # not prepared


def test_prepare_without_gpu_fails_loudly(gg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    b = gg.B200Backend()
    with pytest.raises(gg.GGError) as e:
        b.prepare(gg.BF16, [4], 64, 64, ALIGNED, ALIGNED, ALIGNED)
    assert e.value.code == gg.GG_ERR_CUDA


def test_null_handle_is_rejected(gg):
    lib = gg.load_library()
    assert lib.gg_run(None, None) == gg.GG_ERR_ARG
    assert lib.gg_prepare(None, None, None, None, 0) == gg.GG_ERR_ARG
    st = ctypes.c_uint32(0)
    assert lib.gg_device_status(None, None, ctypes.byref(st)) == gg.GG_ERR_ARG
    lib.gg_release(None)
    lib.gg_destroy(None)


@pytest.mark.parametrize(
    "op,kw,reason",
    [
        ("dgrad", dict(dtype=3), "dtype"),
        ("dgrad", dict(k=100), "k must be a multiple of 8"),
        ("dgrad", dict(w=0), "dy, w and dx must be non-null"),
        ("dgrad", dict(dx=ALIGNED + 4), "16-byte aligned"),
        ("wgrad", dict(x=0), "dy, x and dw must be non-null"),
        ("wgrad", dict(group_m=[0, 0], dw=0), "dy, x and dw must be non-null"),
        ("wgrad", dict(group_m=[4, -2]), "group_m"),
        ("wgrad", dict(group_num_n=True), "group_num * n"),
    ],
)
def test_prepare_grad_refuses_unsupported_arguments(gg, op, kw, reason):
    args = dict(dtype=gg.BF16, group_m=[4, 4], n=64, k=64, dy=ALIGNED, x=ALIGNED, w=ALIGNED, dx=ALIGNED,
                dw=ALIGNED)
    if kw.pop("group_num_n", False):
        args.update(group_m=[1] * 64, n=1 << 26)
    args.update(kw)
    b = gg.B200Backend()
    why = b.prepare_grad(gg.OP_DGRAD if op == "dgrad" else gg.OP_WGRAD, args["dtype"], args["group_m"], args["n"],
                         args["k"], dy_ptr=args["dy"], x_ptr=args["x"], w_ptr=args["w"], dx_ptr=args["dx"],
                         dw_ptr=args["dw"])
    assert reason in why, why
    with pytest.raises(gg.GGError):
        b.run()


def test_prepare_grad_rejects_unknown_op_and_wgrad_split(gg):
    b = gg.B200Backend()
    with pytest.raises(gg.GGError) as e:
        b.prepare_grad(7, gg.BF16, [4], 64, 64, dy_ptr=ALIGNED, x_ptr=ALIGNED, dw_ptr=ALIGNED)
    assert e.value.code == gg.GG_ERR_ARG
    b.set_option("split", 2)
    assert "wgrad" in b.prepare_grad(gg.OP_WGRAD, gg.BF16, [4], 64, 64, dy_ptr=ALIGNED, x_ptr=ALIGNED,
                                     dw_ptr=ALIGNED)
    b.set_option("split", 0)
    b.set_option("stream_k", 1)
    assert "stream-K is not available for wgrad" in b.prepare_grad(gg.OP_WGRAD, gg.BF16, [4], 64, 64, dy_ptr=ALIGNED,
                                                                    x_ptr=ALIGNED, dw_ptr=ALIGNED)


def test_split_and_stream_k_exclude_each_other(gg):
    b = gg.B200Backend()
    b.set_option("split", 2)
    b.set_option("stream_k", 2)
    assert "exclude each other" in b.prepare(gg.BF16, [128], 64, 64, ALIGNED, ALIGNED, ALIGNED)
