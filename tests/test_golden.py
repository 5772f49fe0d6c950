"""Pins the CPU oracle to the reference's own code (no GPU needed).

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs the
reference's bench/bench_main.cpp (compiled unmodified through oracle/ref_shim) on a B200: its
fill_randn made x and w, its make_samples the sample list and its sampled_reference kernel
the fp32 values.

What must hold:
* the sample list is identical (std::mt19937_64(1234), bench/bench_main.cpp:210-227);
* given the reference's input bits, the oracle's fp32 value at each sample is bit-identical
  to the reference kernel's (same fma chain and reduction tree, bench/bench_main.cpp:185-206),
  and its full-output GEMM agrees to fp32 rounding;
* the oracle's host input generator reproduces the reference's device generator except for
  rare elements where the device logf/cospif round differently: at most 0.5% of elements, each
  within 1% relative (+2^-14 absolute) of the reference value.
"""
import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["micro_bf16", "micro_fp16", "tiny_bf16", "pad9003_fp16"]


def load(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    dt = 0 if str(d["dtype"]) == "bf16" else 1
    b, m, n, k = (int(v) for v in d["shape"])
    return d, dt, b, m, n, k


def gen_close(orc, ours, theirs, dt):
    a = orc.to_f32(ours, dt)
    b = orc.to_f32(theirs, dt)
    diff = a != b
    frac = diff.mean()
    ok = np.abs(a - b) <= 1e-2 * np.abs(b) + 2.0 ** -14
    return frac, bool(ok.all())


@pytest.mark.parametrize("name", CASES)
def test_sample_list_identical(orc, name):
    d, dt, b, m, n, k = load(name)
    rows, cols, groups = orc.make_samples([m] * b, n)
    assert np.array_equal(np.stack([rows, cols, groups], 1), d["samples"])


@pytest.mark.parametrize("name", CASES)
def test_generator_matches_reference(orc, name):
    d, dt, b, m, n, k = load(name)
    x, w = orc.make_inputs([m] * b, n, k, dt)
    for ours, theirs in ((x.ravel()[:4096], d["x_head"]), (w.ravel()[:4096], d["w_head"])):
        frac, ok = gen_close(orc, ours, theirs, dt)
        assert frac <= 5e-3 and ok, (frac, ok)
    if "x" in d:
        for ours, theirs in ((x.ravel(), d["x"]), (w.ravel(), d["w"])):
            frac, ok = gen_close(orc, ours, theirs, dt)
            assert frac <= 5e-3 and ok, (frac, ok)


@pytest.mark.parametrize("name", ["micro_bf16", "micro_fp16"])
def test_sampled_reference_bit_exact(orc, name):
    d, dt, b, m, n, k = load(name)
    x = d["x"].reshape(b * m, k)
    w = d["w"].reshape(b, n, k)
    s = d["samples"]
    ref = orc.sampled_ref(x, w, dt, s[:, 0], s[:, 1], s[:, 2])
    assert np.array_equal(ref.view(np.uint32), d["sample_ref"].view(np.uint32))
    # and at every output element
    rows, cols = np.meshgrid(np.arange(b * m), np.arange(n), indexing="ij")
    groups = rows // m
    full = orc.sampled_ref(x, w, dt, rows.ravel(), cols.ravel(), groups.ravel())
    assert np.array_equal(full.view(np.uint32), d["full_ref"].ravel().view(np.uint32))


@pytest.mark.parametrize("name", ["micro_bf16", "micro_fp16"])
def test_full_gemm_matches_reference_values(orc, name):
    d, dt, b, m, n, k = load(name)
    x = d["x"].reshape(b * m, k)
    w = d["w"].reshape(b, n, k)
    full = orc.grouped_gemm_f32(x, w, [m] * b, dt)
    ref = d["full_ref"]
    assert np.abs(full - ref).max() <= 1e-6 * np.abs(ref).max()


@pytest.mark.parametrize("name", ["tiny_bf16", "pad9003_fp16"])
def test_reference_values_on_oracle_inputs(orc, name):
    # The larger fixtures keep only digests of the reference's inputs; on the oracle's own
    # inputs (which differ in a handful of elements) the sampled values satisfy the pass rule.
    d, dt, b, m, n, k = load(name)
    x, w = orc.make_inputs([m] * b, n, k, dt)
    s = d["samples"]
    ref = orc.sampled_ref(x, w, dt, s[:, 0], s[:, 1], s[:, 2])
    bad, mx = orc.check(ref, d["sample_ref"])
    assert bad == 0 and mx < 0.05, (bad, mx)
    assert len(str(d["x_sha256"])) == 64 and hashlib.sha256(b"").hexdigest() != str(d["x_sha256"])
