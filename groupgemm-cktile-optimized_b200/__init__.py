"""Python binding of the B200 grouped-GEMM backend (ctypes over include/gg_b200.h).

The product is the C ABI in lib/libgg_b200.so; this module is the ctypes stub a Python caller
binds it with. `B200Backend` mirrors the reference's `tunemax::Backend`
(common/backend.hpp:62-79): prepare() is untimed and returns "" or an N/A reason, run()
enqueues one grouped GEMM, release() frees what prepare() allocated, detail() describes the
kernel chosen. Device buffers are passed as raw pointers (e.g. torch's `data_ptr()`), streams
as raw `cudaStream_t` handles (e.g. `torch.cuda.current_stream().cuda_stream`).

There is no fallback: if the library is missing this module raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libgg_b200.so")
# The same C ABI with the kernel's bounds checks compiled in (-DGG_DEBUG): load it with
# load_library(DEBUG_LIB_PATH) into a module of its own (see tests/test_gpu_debug_build.py).
DEBUG_LIB_PATH = os.path.join(HERE, "lib", "libgg_b200_debug.so")

BF16, FP16 = 0, 1
DTYPES = {"bf16": BF16, "fp16": FP16}

GG_OK, GG_NOT_SUPPORTED, GG_ERR_ARG, GG_ERR_CUDA, GG_ERR_DEVICE = 0, 1, -1, -2, -3

# Variant ids accepted by set_option("variant", v).
VARIANT_AUTO, VARIANT_2CTA_256x256, VARIANT_1CTA_128x256, VARIANT_1CTA_128x128 = -1, 0, 1, 2


class GGProblem(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("group_num", ctypes.c_int32),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("group_m", ctypes.POINTER(ctypes.c_int64)),
        ("x", ctypes.c_void_p),
        ("w", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]


# Backward operations accepted by B200Backend.prepare_grad (enum gg_op).
OP_FORWARD, OP_DGRAD, OP_WGRAD = 0, 1, 2


class GGGradProblem(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("group_num", ctypes.c_int32),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("group_m", ctypes.POINTER(ctypes.c_int64)),
        ("dy", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("w", ctypes.c_void_p),
        ("dx", ctypes.c_void_p),
        ("dw", ctypes.c_void_p),
    ]


# Every symbol include/gg_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "gg_abi_version": (ctypes.c_int, []),
    "gg_create": (ctypes.c_void_p, []),
    "gg_name": (ctypes.c_char_p, [ctypes.c_void_p]),
    "gg_prepare": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GGProblem), ctypes.c_void_p,
                                  ctypes.c_char_p, ctypes.c_size_t]),
    "gg_prepare_grad": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GGGradProblem), ctypes.c_int32,
                                       ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "gg_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "gg_release": (None, [ctypes.c_void_p]),
    "gg_detail": (ctypes.c_char_p, [ctypes.c_void_p]),
    "gg_last_error": (ctypes.c_char_p, [ctypes.c_void_p]),
    "gg_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "gg_set_option": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64]),
    "gg_destroy": (None, [ctypes.c_void_p]),
    "gg_expert_shard": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "gg_run_noalloc": (ctypes.c_int, [ctypes.POINTER(GGProblem), ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32),
                                      ctypes.c_char_p, ctypes.c_size_t]),
}

_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libgg_b200.so and attach signatures. Raises if it was not built."""
    global _lib
    if _lib is not None and path == LIB_PATH:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python __graft_entry__.py build` "
                           "(there is no CPU or library fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path == LIB_PATH:
        _lib = lib
    return lib


class GGError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gg error {code}: {msg}")
        self.code = code


def expert_shard(group_num: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous expert range [g0, g1) of `rank` (host arithmetic of gg_expert_shard)."""
    lib = load_library()
    g0, g1 = ctypes.c_int32(), ctypes.c_int32()
    rc = lib.gg_expert_shard(group_num, world, rank, ctypes.byref(g0), ctypes.byref(g1))
    if rc != GG_OK:
        raise GGError(rc, "bad expert_shard arguments")
    return g0.value, g1.value


class B200Backend:
    """tunemax::Backend over the C ABI (common/backend.hpp:62-79)."""

    def __init__(self) -> None:
        self._lib = load_library()
        self._h = self._lib.gg_create()
        if not self._h:
            raise MemoryError("gg_create failed")
        self._group_m = None  # keep the host array alive while prepared

    def __del__(self) -> None:
        h, self._h = getattr(self, "_h", None), None
        if h and getattr(self, "_lib", None) is not None:
            self._lib.gg_destroy(h)

    def name(self) -> str:
        return self._lib.gg_name(self._h).decode()

    def set_option(self, key: str, value: int) -> None:
        rc = self._lib.gg_set_option(self._h, key.encode(), int(value))
        if rc != GG_OK:
            raise GGError(rc, self.last_error())

    def prepare(self, dtype: int, group_m: Sequence[int], n: int, k: int, x_ptr: int, w_ptr: int,
                out_ptr: int, stream: int = 0) -> str:
        """Returns "" when ready or the reason the shape is not supported (N/A).
        Raises GGError on a CUDA or argument error."""
        gm = (ctypes.c_int64 * len(group_m))(*[int(m) for m in group_m])
        self._group_m = gm
        prob = GGProblem(int(dtype), len(group_m), int(n), int(k), gm, ctypes.c_void_p(x_ptr or None),
                         ctypes.c_void_p(w_ptr or None), ctypes.c_void_p(out_ptr or None))
        why = ctypes.create_string_buffer(256)
        rc = self._lib.gg_prepare(self._h, ctypes.byref(prob), ctypes.c_void_p(stream or None), why, 256)
        if rc == GG_OK:
            return ""
        if rc == GG_NOT_SUPPORTED:
            return why.value.decode() or "not supported"
        raise GGError(rc, self.last_error())

    def prepare_grad(self, op: int, dtype: int, group_m: Sequence[int], n: int, k: int, dy_ptr: int = 0,
                     x_ptr: int = 0, w_ptr: int = 0, dx_ptr: int = 0, dw_ptr: int = 0, stream: int = 0) -> str:
        """Prepare a backward grouped GEMM: OP_DGRAD (dx = dy @ w[g], needs dy, w, dx) or OP_WGRAD
        (dw[g] = dy[g]^T @ x[g], needs dy, x, dw). Then run() launches it. Returns "" or the N/A
        reason; raises GGError on a CUDA or argument error."""
        gm = (ctypes.c_int64 * len(group_m))(*[int(m) for m in group_m])
        self._group_m = gm
        vp = lambda v: ctypes.c_void_p(v or None)  # noqa: E731
        prob = GGGradProblem(int(dtype), len(group_m), int(n), int(k), gm, vp(dy_ptr), vp(x_ptr), vp(w_ptr),
                             vp(dx_ptr), vp(dw_ptr))
        why = ctypes.create_string_buffer(256)
        rc = self._lib.gg_prepare_grad(self._h, ctypes.byref(prob), int(op), vp(stream), why, 256)
        if rc == GG_OK:
            return ""
        if rc == GG_NOT_SUPPORTED:
            return why.value.decode() or "not supported"
        raise GGError(rc, self.last_error())

    def run(self, stream: int = 0) -> None:
        rc = self._lib.gg_run(self._h, ctypes.c_void_p(stream or None))
        if rc != GG_OK:
            raise GGError(rc, self.last_error())

    def release(self) -> None:
        self._lib.gg_release(self._h)

    def detail(self) -> str:
        return self._lib.gg_detail(self._h).decode()

    def last_error(self) -> str:
        return self._lib.gg_last_error(self._h).decode()

    def device_status(self, stream: int = 0) -> int:
        """Synchronise, read and clear the kernel's status word (0 = every wait finished)."""
        st = ctypes.c_uint32(0)
        rc = self._lib.gg_device_status(self._h, ctypes.c_void_p(stream or None), ctypes.byref(st))
        if rc not in (GG_OK, GG_ERR_DEVICE):
            raise GGError(rc, self.last_error())
        return st.value


def run_noalloc(dtype: int, group_m: Sequence[int], n: int, k: int, x_ptr: int, w_ptr: int, out_ptr: int,
                stream: int = 0, wait: bool = False) -> tuple[int, str, int]:
    """gg_run_noalloc: one grouped GEMM for callers that cannot allocate device memory.

    The library keeps its small per-call scratch (group offsets and status word, at most 1024
    groups) in a fixed device array instead of allocating it, so nothing is allocated here.
    Returns (return code, reason or error text, status word when `wait`, else 0). The status
    word is shared and sticky: a waited call reports (and clears) the first bounded-wait timeout
    of any call since the last waited one. Calls that can overlap on the GPU share that array and
    race; calls in order on one stream are fine."""
    lib = load_library()
    gm = (ctypes.c_int64 * len(group_m))(*[int(m) for m in group_m])
    prob = GGProblem(int(dtype), len(group_m), int(n), int(k), gm, ctypes.c_void_p(x_ptr or None),
                     ctypes.c_void_p(w_ptr or None), ctypes.c_void_p(out_ptr or None))
    why = ctypes.create_string_buffer(256)
    st = ctypes.c_uint32(0)
    rc = lib.gg_run_noalloc(ctypes.byref(prob), ctypes.c_void_p(stream or None),
                            ctypes.byref(st) if wait else None, why, 256)
    return rc, why.value.decode(), st.value


def make_b200_backend() -> B200Backend:
    """Factory beside the reference's make_ck_tile_backend() (common/backend.hpp:81-83)."""
    return B200Backend()
