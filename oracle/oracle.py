"""ctypes/numpy front end of the CPU oracle (lib/liboracle.so, built from gg_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg, as the checker. The product path never imports it.

Each function cites the reference code it restates (paths inside the reference project).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "liboracle.so")
REF_HARNESS = os.path.join(HERE, "_ref", "ref_harness")

_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `python oracle/build.py`")
        _lib = ctypes.CDLL(LIB_PATH)
        sig = {
            "orc_hw_threads": (ctypes.c_int, []),
            "orc_splitmix64": (ctypes.c_uint64, [ctypes.c_uint64]),
            "orc_randn_at": (ctypes.c_float, [ctypes.c_uint64, ctypes.c_uint64]),
            "orc_f32_to_16": (ctypes.c_uint16, [ctypes.c_float, ctypes.c_int]),
            "orc_16_to_f32": (ctypes.c_float, [ctypes.c_uint16, ctypes.c_int]),
            "orc_to_f32": (None, [_P, _P, _I64, ctypes.c_int]),
            "orc_from_f32": (None, [_P, _P, _I64, ctypes.c_int]),
            "orc_fill_randn": (None, [_P, _I64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]),
            "orc_grouped_gemm_f32": (None, [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, _I64, _I64,
                                            ctypes.c_int, ctypes.c_int, _I64, ctypes.c_int]),
            "orc_make_samples": (_I64, [ctypes.c_int, _P, _I64, _P, _P, _P, _I64]),
            "orc_sampled_ref": (None, [_P, _P, ctypes.c_int, _I64, _I64, _P, _P, _P, _I64, _P, ctypes.c_int]),
            "orc_check": (_I64, [_P, _P, _I64, ctypes.POINTER(ctypes.c_double)]),
            "orc_check16": (_I64, [_P, _P, _I64, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_int64)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(_lib, name)
            f.restype = res
            f.argtypes = args
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def hw_threads() -> int:
    return int(lib().orc_hw_threads())


def fill_randn(n: int, seed: int, dtype: int, threads: int = 0) -> np.ndarray:
    """16-bit patterns of the reference input fill (bench/bench_main.cpp:160-176, 295-298)."""
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_randn(_ptr(out), n, seed, dtype, threads)
    return out


def to_f32(bits: np.ndarray, dtype: int) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    lib().orc_to_f32(_ptr(bits), _ptr(out), bits.size, dtype)
    return out


def from_f32(vals: np.ndarray, dtype: int) -> np.ndarray:
    vals = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.empty(vals.shape, dtype=np.uint16)
    lib().orc_from_f32(_ptr(vals), _ptr(out), vals.size, dtype)
    return out


def make_inputs(group_m, n: int, k: int, dtype: int, threads: int = 0):
    """x [sum(M), k] (seed 1) and w [G, n, k] (seed 2) as 16-bit patterns
    (bench/bench_main.cpp:450-457)."""
    total = int(sum(group_m))
    x = fill_randn(total * k, 1, dtype, threads).reshape(total, k)
    w = fill_randn(len(group_m) * n * k, 2, dtype, threads).reshape(len(group_m), n, k)
    return x, w


def grouped_gemm_f32(x: np.ndarray, w: np.ndarray, group_m, dtype: int, groups=None,
                     max_rows: int = -1, threads: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """fp32 out [sum(M), n] of the grouped GEMM (the reference op's fp32 math,
    bench/bench_main.cpp:185-206, over ck_kernel/ck_grouped_gemm.cpp:166-188's group layout).
    Only groups in `groups` = (g0, g1) and the first `max_rows` rows of each are computed."""
    gm = np.ascontiguousarray(group_m, dtype=np.int64)
    G, n, k = w.shape
    total = int(gm.sum())
    if out is None:
        out = np.zeros((total, n), dtype=np.float32)
    g0, g1 = groups if groups is not None else (0, G)
    lib().orc_grouped_gemm_f32(_ptr(np.ascontiguousarray(x)), _ptr(np.ascontiguousarray(w)), _ptr(out),
                               dtype, G, _ptr(gm), n, k, g0, g1, max_rows, threads)
    return out


def make_samples(group_m, n: int):
    """(rows, cols, groups) of bench/bench_main.cpp:210-227."""
    gm = np.ascontiguousarray(group_m, dtype=np.int64)
    cap = 260 * len(gm)
    rows = np.empty(cap, np.int64)
    cols = np.empty(cap, np.int64)
    grps = np.empty(cap, np.int64)
    cnt = lib().orc_make_samples(len(gm), _ptr(gm), n, _ptr(rows), _ptr(cols), _ptr(grps), cap)
    return rows[:cnt].copy(), cols[:cnt].copy(), grps[:cnt].copy()


def sampled_ref(x: np.ndarray, w: np.ndarray, dtype: int, rows, cols, groups, threads: int = 0) -> np.ndarray:
    """fp32 reference values at the samples, in the reference kernel's summation order
    (bench/bench_main.cpp:185-206)."""
    G, n, k = w.shape
    rows = np.ascontiguousarray(rows, np.int64)
    cols = np.ascontiguousarray(cols, np.int64)
    groups = np.ascontiguousarray(groups, np.int64)
    ref = np.empty(rows.size, np.float32)
    lib().orc_sampled_ref(_ptr(np.ascontiguousarray(x)), _ptr(np.ascontiguousarray(w)), dtype, n, k,
                          _ptr(rows), _ptr(cols), _ptr(groups), rows.size, _ptr(ref), threads)
    return ref


def check(got: np.ndarray, ref: np.ndarray):
    """Pass rule of bench/bench_main.cpp:263-270 -> (mismatches, max_abs)."""
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    mx = ctypes.c_double(0)
    bad = lib().orc_check(_ptr(got), _ptr(ref), got.size, ctypes.byref(mx))
    return int(bad), float(mx.value)


def check16(got_bits: np.ndarray, ref: np.ndarray, dtype: int):
    """Pass rule over 16-bit outputs -> (mismatches, max_abs, first_bad_index)."""
    got_bits = np.ascontiguousarray(got_bits, np.uint16)
    ref = np.ascontiguousarray(ref, np.float32)
    mx = ctypes.c_double(0)
    first = ctypes.c_int64(-1)
    bad = lib().orc_check16(_ptr(got_bits), _ptr(ref), got_bits.size, dtype, ctypes.byref(mx), ctypes.byref(first))
    return int(bad), float(mx.value), int(first.value)


# ---- backward grouped GEMMs ---------------------------------------------------------------
# The reference benchmarks the forward op only. Its vendored Primus-Turbo grouped GEMM defines
# the two backward calls of the same MoE layer (third_party/primus_turbo/kernels/
# hipblaslt_grouped_gemm.cu:80-96 shape rules, :199-240 per-group arguments): grad_a = grad_c x b
# (non-transA) and grad_b = a^T x grad_c (transA), with an expert that received no tokens given a
# zero gradient (:201-214). These restate that math in float64 on the decoded 16-bit inputs and
# return float32, the precision the forward oracle's pass rule compares against.

def make_grad_inputs(group_m, n: int, k: int, dtype: int, threads: int = 0):
    """dy [sum(M), n] (seed 3) plus x (seed 1) and w (seed 2) as in make_inputs, as 16-bit patterns.
    The reference has no backward harness; seed 3 continues its seed numbering."""
    x, w = make_inputs(group_m, n, k, dtype, threads)
    dy = fill_randn(int(sum(group_m)) * n, 3, dtype, threads).reshape(int(sum(group_m)), n)
    return dy, x, w


def grouped_dgrad_f32(dy: np.ndarray, w: np.ndarray, group_m, dtype: int) -> np.ndarray:
    """dx [sum(M), k] = dy[rows of g] @ w[g] (hipblaslt_grouped_gemm.cu:91-95, non-transA)."""
    G, n, k = w.shape
    dyf = to_f32(dy, dtype).astype(np.float64).reshape(-1, n)
    wf = to_f32(w, dtype).astype(np.float64)
    out = np.zeros((dyf.shape[0], k), np.float32)
    r0 = 0
    for g, m in enumerate(group_m):
        if m:
            out[r0:r0 + m] = dyf[r0:r0 + m] @ wf[g]
        r0 += int(m)
    return out


def grouped_wgrad_f32(dy: np.ndarray, x: np.ndarray, group_m, dtype: int) -> np.ndarray:
    """dw [G, n, k], dw[g] = dy[rows of g]^T @ x[rows of g]; zero for an empty group
    (hipblaslt_grouped_gemm.cu:82-90 transA, :201-214)."""
    n = dy.shape[-1]
    k = x.shape[-1]
    dyf = to_f32(dy, dtype).astype(np.float64).reshape(-1, n)
    xf = to_f32(x, dtype).astype(np.float64).reshape(-1, k)
    out = np.zeros((len(group_m), n, k), np.float32)
    r0 = 0
    for g, m in enumerate(group_m):
        if m:
            out[g] = dyf[r0:r0 + m].T @ xf[r0:r0 + m]
        r0 += int(m)
    return out
