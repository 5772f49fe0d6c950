"""Generate the golden fixtures in this directory from the reference's own code.

Runs oracle/_ref/ref_harness (the reference's bench/bench_main.cpp compiled unmodified through
oracle/ref_shim) on a GPU: its fill_randn produces x/w, its make_samples the sample list, its
sampled_reference kernel the fp32 reference values. Each case is packed into one compressed
.npz:

  small cases (full=1): x, w (uint16 bit patterns), samples (int64 [S,3] row/col/group),
                        sample_ref (float32 [S]), full_ref (float32 [sum(M), N])
  larger cases        : x_sha256, w_sha256 (of the raw little-endian bit patterns), x_head,
                        w_head (first 4096 elements), samples, sample_ref

Usage (on a machine with an sm_100 GPU):  python tests/golden/make_golden.py OUT_DIR
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")

# name, dtype, B, M, N, K, full
CASES = [
    ("micro_bf16", "bf16", 2, 40, 72, 136, True),
    ("micro_fp16", "fp16", 3, 33, 40, 72, True),
    ("tiny_bf16", "bf16", 4, 256, 512, 384, False),      # BASELINE config T
    ("pad9003_fp16", "fp16", 2, 300, 1000, 2048, False),  # shapes/pad_test.csv row 9003
]


def main(out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    for name, dt, b, m, n, k, full in CASES:
        with tempfile.TemporaryDirectory() as tmp:
            cmd = [HARNESS, "golden", tmp, dt, str(b), str(m), str(n), str(k)] + (["full"] if full else [])
            subprocess.run(cmd, check=True)
            x = np.fromfile(os.path.join(tmp, "x.u16"), np.uint16)
            w = np.fromfile(os.path.join(tmp, "w.u16"), np.uint16)
            samples = np.fromfile(os.path.join(tmp, "samples.i64"), np.int64).reshape(-1, 3)
            sref = np.fromfile(os.path.join(tmp, "sample_ref.f32"), np.float32)
            arrays = dict(dtype=np.array(dt), shape=np.array([b, m, n, k], np.int64), samples=samples,
                          sample_ref=sref,
                          x_sha256=np.array(hashlib.sha256(x.tobytes()).hexdigest()),
                          w_sha256=np.array(hashlib.sha256(w.tobytes()).hexdigest()),
                          x_head=x[:4096].copy(), w_head=w[:4096].copy())
            if full:
                arrays["x"] = x
                arrays["w"] = w
                arrays["full_ref"] = np.fromfile(os.path.join(tmp, "full_ref.f32"), np.float32).reshape(b * m, n)
            np.savez_compressed(os.path.join(out_dir, name + ".npz"), **arrays)
            print("wrote", name, {kk: getattr(v, "shape", None) for kk, v in arrays.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
