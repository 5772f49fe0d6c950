"""The bounds-checked debug build (lib/libgg_b200_debug.so, compiled with -DGG_DEBUG): before each
global store, workspace access and arrival-counter access, and on every decoded tile, the kernel
checks the index against the problem's bounds; a failed check records 0x2000 | site in the device
status word and skips the access (nothing traps). The release build has none of these checks.

* Seeded random cases of the fuzz suite (every operation, split-K, stream-K, tile widths, dynamic
  dispatch, split launches) run through the debug build: every check holds (status 0) and the
  outputs match the oracle.
* The test-only option test_bounds declares the output one row short, so the debug build must
  find the last row's stores out of bounds, skip them and report site 2, while every other row is
  stored correctly. No access outside the real buffers happens.
"""
import importlib.util
import os

import numpy as np
import pytest

from conftest import PKG_DIR

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


@pytest.fixture(scope="module")
def ggd():
    """A second instance of the binding module, bound to the debug library."""
    spec = importlib.util.spec_from_file_location("gg_b200_debug", os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod._lib = mod.load_library(mod.DEBUG_LIB_PATH)
    return mod


@pytest.mark.parametrize("seed", range(24))
def test_fuzz_cases_pass_every_check(ggd, orc, seed):
    _torch()
    import test_gpu_fuzz as fz

    fz.check_case(ggd, orc, fz.draw_case(np.random.default_rng(1000 + seed)))


@pytest.mark.parametrize("seed", range(8))
def test_stream_k_cases_pass_every_check(ggd, orc, seed):
    _torch()
    import test_gpu_fuzz as fz

    fz.check_case(ggd, orc, fz.draw_case_stream_k(np.random.default_rng(5000 + seed)))


def test_split_launch_passes_every_check(ggd, orc):
    torch = _torch()
    group_m, n, k = [1, 64, 0, 65, 128, 129, 356, 640, 300], 776, 520
    x, w = orc.make_inputs(group_m, n, k, 0)
    ref = orc.grouped_gemm_f32(x, w, group_m, 0)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    out = torch.zeros(sum(group_m) * n, dtype=torch.int16, device="cuda")
    b = ggd.B200Backend()
    b.set_option("variant", 0)
    b.set_option("tail_launch", 1)
    s = torch.cuda.current_stream().cuda_stream
    assert b.prepare(0, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    assert "+tail" in b.detail()
    b.run(s)
    assert b.device_status(s) == 0
    assert orc.check16(out.cpu().numpy().view(np.uint16).reshape(-1, n), ref, 0)[0] == 0


def test_debug_build_reports_and_skips_a_store_past_the_declared_output(ggd, orc):
    torch = _torch()
    group_m, n, k = [300, 200], 512, 1024  # K >= 1024: stores straight from registers
    x, w = orc.make_inputs(group_m, n, k, 0)
    ref = orc.grouped_gemm_f32(x, w, group_m, 0)
    rows = sum(group_m)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    out = torch.zeros(rows * n, dtype=torch.int16, device="cuda")
    b = ggd.B200Backend()
    b.set_option("test_bounds", 1)
    b.set_option("store", 1)
    s = torch.cuda.current_stream().cuda_stream
    assert b.prepare(0, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    st = b.device_status(s)
    assert st == 0x2002, hex(st)
    got = out.cpu().numpy().view(np.uint16).reshape(rows, n)
    assert orc.check16(got[:-1], ref[:-1], 0)[0] == 0  # every declared row stored
    assert not got[-1].any()  # the row past the declared output was skipped
    # the handle works normally again once the status is read
    b.set_option("test_bounds", 0)
    assert b.prepare(0, group_m, n, k, xd.data_ptr(), wd.data_ptr(), out.data_ptr(), s) == ""
    b.run(s)
    assert b.device_status(s) == 0
    assert orc.check16(out.cpu().numpy().view(np.uint16).reshape(rows, n), ref, 0)[0] == 0
