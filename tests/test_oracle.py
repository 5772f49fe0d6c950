"""CPU tests of the oracle itself (no GPU).

The oracle restates the reference harness's arithmetic (bench/bench_main.cpp). These tests check
each piece against an independent statement: torch's dtype conversions, a pure-Python
std::mt19937_64, numpy float64 GEMMs, and the pass rule's edge cases.
"""
import numpy as np
import pytest
import torch


def test_bf16_fp16_conversions_match_torch(orc):
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(50000).astype(np.float32) * s for s in (1e-6, 1, 1e3, 7e4)])
    v = np.concatenate([v, np.array([0.0, -0.0, 65504, 65519, 65520, -65520, 6e-8, 3e-8, 1e-9,
                                     np.inf, -np.inf], np.float32)])
    for dt, tdt in ((0, torch.bfloat16), (1, torch.float16)):
        want = torch.from_numpy(v).to(tdt).view(torch.int16).numpy().view(np.uint16)
        got = orc.from_f32(v, dt)
        assert np.array_equal(got, want), f"dtype {dt}: {np.flatnonzero(got != want)[:5]}"
        back = orc.to_f32(got, dt)
        tback = torch.from_numpy(got.view(np.int16)).view(tdt).float().numpy()
        assert np.array_equal(back, tback)


def test_nan_survives_conversion(orc):
    v = np.array([np.nan], np.float32)
    for dt in (0, 1):
        assert np.isnan(orc.to_f32(orc.from_f32(v, dt), dt)[0])


def test_generator_is_standard_normal_and_deterministic(orc):
    a = orc.to_f32(orc.fill_randn(1 << 18, 1, 0), 0)
    b = orc.to_f32(orc.fill_randn(1 << 18, 1, 0), 0)
    c = orc.to_f32(orc.fill_randn(1 << 18, 2, 0), 0)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    # threads do not change the values
    assert np.array_equal(orc.fill_randn(100003, 7, 1, threads=1), orc.fill_randn(100003, 7, 1, threads=5))


def test_generator_matches_python_restatement(orc):
    # Element i from splitmix64 + Box-Muller in plain Python (bench/bench_main.cpp:160-176).
    import math
    import struct

    def f32(x):
        return struct.unpack("f", struct.pack("f", x))[0]

    M = (1 << 64) - 1

    def splitmix64(x):
        x = (x + 0x9E3779B97F4A7C15) & M
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
        return x ^ (x >> 31)

    for seed in (1, 2):
        vals = orc.fill_randn(64, seed, 0)
        for i in range(64):
            r = splitmix64(seed ^ ((i * 0x2545F4914F6CDD1D) & M))
            u1 = f32(f32(float(r >> 40) + 1.0) * f32(1.0 / 16777217.0))
            u2 = f32(float((r >> 16) & 0xFFFFFF) * f32(1.0 / 16777216.0))
            v = f32(f32(math.sqrt(-2.0 * math.log(u1))) * f32(math.cos(math.pi * f32(2.0 * u2))))
            want = torch.tensor([v], dtype=torch.float32).to(torch.bfloat16).view(torch.int16).item() & 0xFFFF
            assert vals[i] == want, (seed, i)


class MT19937_64:
    """std::mt19937_64 written out from its published definition (Matsumoto & Nishimura)."""

    def __init__(self, seed):
        self.mt = [0] * 312
        self.mt[0] = seed & 0xFFFFFFFFFFFFFFFF
        for i in range(1, 312):
            self.mt[i] = (6364136223846793005 * (self.mt[i - 1] ^ (self.mt[i - 1] >> 62)) + i) & 0xFFFFFFFFFFFFFFFF
        self.i = 312

    def __call__(self):
        if self.i >= 312:
            for j in range(312):
                x = (self.mt[j] & 0xFFFFFFFF80000000) | (self.mt[(j + 1) % 312] & 0x7FFFFFFF)
                xa = x >> 1
                if x & 1:
                    xa ^= 0xB5026F5AA96619E9
                self.mt[j] = self.mt[(j + 156) % 312] ^ xa
            self.i = 0
        y = self.mt[self.i]
        self.i += 1
        y ^= (y >> 29) & 0x5555555555555555
        y ^= (y << 17) & 0x71D67FFFEDA60000
        y ^= (y << 37) & 0xFFF7EEE000000000
        y ^= y >> 43
        return y


def test_mt19937_64_known_answer():
    # The C++ standard fixes the 10000th output of a default-seeded std::mt19937_64.
    g = MT19937_64(5489)
    for _ in range(9999):
        g()
    assert g() == 9981545732273789042


def test_make_samples_rule(orc):
    group_m = [5, 0, 300, 1]
    n = 77
    rows, cols, groups = orc.make_samples(group_m, n)
    assert len(rows) == 3 * 260
    rng = MT19937_64(1234)
    idx, row0 = 0, 0
    for g, m in enumerate(group_m):
        if m > 0:
            corners = [(row0, 0), (row0, n - 1), (row0 + m - 1, 0), (row0 + m - 1, n - 1)]
            for (r, c) in corners:
                assert (rows[idx], cols[idx], groups[idx]) == (r, c, g)
                idx += 1
            for _ in range(256):
                r = row0 + rng() % m
                c = rng() % n
                assert (rows[idx], cols[idx], groups[idx]) == (r, c, g)
                idx += 1
        row0 += m


def _np_ref(x, w, group_m, dt, orc):
    xf = orc.to_f32(x, dt).astype(np.float64)
    wf = orc.to_f32(w, dt).astype(np.float64)
    out, r0 = [], 0
    for g, m in enumerate(group_m):
        out.append(xf[r0:r0 + m] @ wf[g].T)
        r0 += m
    return np.concatenate(out) if out else np.zeros((0, w.shape[1]))


@pytest.mark.parametrize("dt", [0, 1])
def test_full_gemm_matches_float64(orc, dt):
    group_m = [3, 0, 67, 16]
    n, k = 40, 136
    x, w = orc.make_inputs(group_m, n, k, dt)
    out = orc.grouped_gemm_f32(x, w, group_m, dt)
    ref = _np_ref(x, w, group_m, dt, orc)
    assert np.allclose(out, ref, rtol=1e-5, atol=1e-4)


def test_partial_gemm_groups_and_rows(orc):
    group_m = [10, 20, 30]
    n, k = 16, 24
    x, w = orc.make_inputs(group_m, n, k, 0)
    full = orc.grouped_gemm_f32(x, w, group_m, 0)
    part = orc.grouped_gemm_f32(x, w, group_m, 0, groups=(1, 3), max_rows=7)
    assert np.all(part[:10] == 0)
    assert np.array_equal(part[10:17], full[10:17])
    assert np.all(part[17:30] == 0)
    assert np.array_equal(part[30:37], full[30:37])


def test_sampled_ref_matches_full(orc):
    group_m = [256] * 4
    n, k = 512, 384
    x, w = orc.make_inputs(group_m, n, k, 0)
    full = orc.grouped_gemm_f32(x, w, group_m, 0)
    rows, cols, groups = orc.make_samples(group_m, n)
    s = orc.sampled_ref(x, w, 0, rows, cols, groups)
    assert np.allclose(s, full[rows, cols], rtol=1e-5, atol=1e-4)


def test_check_rule(orc):
    ref = np.array([0.0, 100.0, -5.0, 1.0], np.float32)
    ok = np.array([0.0099, 100.0 + 1.009, -5.0 - 0.059, 1.0], np.float32)
    bad, mx = orc.check(ok, ref)
    assert bad == 0 and abs(mx - 1.009) < 1e-3
    worse = ok.copy()
    worse[1] = 100.0 + 1.02
    assert orc.check(worse, ref)[0] == 1
    nan = ok.copy()
    nan[0] = np.nan
    bad, mx = orc.check(nan, ref)
    assert bad == 1 and mx == np.inf


@pytest.mark.parametrize("dt", [0, 1])
def test_backward_oracle_matches_forward_oracle_on_transposed_operands(orc, dt):
    # dgrad: dx = dy @ w[g] is the forward op with weights w[g]^T ([G, k, n]).
    # wgrad: dw[g] = dy_g^T @ x_g is the forward op of one group with x' = dy_g^T, w' = x_g^T.
    group_m = [5, 0, 70, 33]
    n, k = 48, 40
    dy, x, w = orc.make_grad_inputs(group_m, n, k, dt)
    dx = orc.grouped_dgrad_f32(dy, w, group_m, dt)
    wt = np.ascontiguousarray(np.transpose(w, (0, 2, 1)))
    assert np.allclose(dx, orc.grouped_gemm_f32(dy, wt, group_m, dt), rtol=1e-5, atol=1e-4)
    dw = orc.grouped_wgrad_f32(dy, x, group_m, dt)
    assert dw.shape == (4, n, k)
    r0 = 0
    for g, m in enumerate(group_m):
        if m == 0:
            assert np.all(dw[g] == 0)
        else:
            xt = np.ascontiguousarray(dy[r0:r0 + m].T)
            wg = np.ascontiguousarray(x[r0:r0 + m].T)[None]
            assert np.allclose(dw[g], orc.grouped_gemm_f32(xt, wg, [n], dt), rtol=1e-5, atol=1e-4)
        r0 += m


def test_grad_inputs_are_deterministic(orc):
    a = orc.make_grad_inputs([3, 4], 16, 8, 0)
    b = orc.make_grad_inputs([3, 4], 16, 8, 0)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
    assert a[0].shape == (7, 16) and a[1].shape == (7, 8) and a[2].shape == (2, 16, 8)
