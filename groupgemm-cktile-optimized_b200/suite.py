"""Suite workflow around the C++ harness (lib/gg_bench): run a shapes CSV one process per case
over the GPUs of a box, merge the per-case results CSVs, and compare two backends.

    python suite.py run SHAPES.csv OUT.csv [--ngpu N] [--timeout S] [-- gg_bench args ...]
    python suite.py compare RESULTS.csv|DIR ... [--ours b200] [--other cublas_loop]

`run` is the counterpart of the reference's scripts/run_parallel.sh:10-30. Every case runs in a
process of its own (`gg_bench --only ID`), with a time limit; cases are dealt round-robin to the
GPUs, one worker per GPU running its cases one after another, and all backends of a case run in
that one process on the same GPU, so a comparison never mixes GPUs. The merged CSV has the
harness's header and its rows in TestID order. As the reference notes, cases running on every
GPU of a box at once share its power and cooling; report numbers from --ngpu 1.

`compare` is the counterpart of scripts/compare.py:4-28: over the cases where our backend
PASSes and the other PASSes (or was timed unchecked, SKIP), the number of cases where ours is
faster, the geomean of the time ratio (other / ours), the summed times, the mean TFLOPS, the
worst cases for ours, and the cases where any row is neither PASS nor SKIP.

A results CSV also serves as a shapes file (its TestID,Case,B,M,N,K columns, one case per
TestID), so a committed results file is enough to re-run its cases.
"""
from __future__ import annotations

import argparse
import csv
import glob
import math
import os
import subprocess
import sys
import tempfile
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
GG_BENCH = os.path.join(HERE, "lib", "gg_bench")
SHAPE_COLS = ("TestID", "Case", "B", "M", "N", "K")


def read_shapes(path: str) -> list[dict]:
    """Cases of a shapes or results CSV: one dict per TestID (first row wins), in file order."""
    seen, cases = set(), []
    with open(path, newline="") as f:
        for row in csv.DictReader(f):
            tid = int(row["TestID"])
            if tid not in seen:
                seen.add(tid)
                cases.append({c: row[c] for c in SHAPE_COLS})
    return cases


def write_shapes(cases: list[dict], path: str) -> None:
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=SHAPE_COLS)
        w.writeheader()
        w.writerows(cases)


def merge_results(paths: list[str], out: str) -> int:
    """Concatenate results CSVs (one header) with rows ordered by TestID; returns the row count."""
    header, rows = None, []
    for p in paths:
        with open(p, newline="") as f:
            r = csv.reader(f)
            h = next(r, None)
            if h is None:
                continue
            if header is None:
                header = h
            elif h != header:
                raise ValueError(f"{p}: header differs from the first file's")
            rows += [row for row in r if row]
    tid = header.index("TestID") if header else 0
    rows.sort(key=lambda row: int(row[tid]))
    with open(out, "w", newline="") as f:
        w = csv.writer(f)
        if header:
            w.writerow(header)
        w.writerows(rows)
    return len(rows)


def run_suite(shapes: str, out: str, ngpu: int = 1, timeout_s: float = 300.0, extra: list[str] | None = None,
              binary: str = GG_BENCH, log=sys.stderr) -> list[str]:
    """One gg_bench process per case, cases dealt round-robin over `ngpu` GPUs (CUDA_VISIBLE_DEVICES),
    each process limited to `timeout_s`. Writes the merged results CSV to `out`; returns the
    failures ("case ID: ..." lines)."""
    extra = list(extra or [])
    cases = read_shapes(shapes)
    failures: list[str] = []
    lock = threading.Lock()
    with tempfile.TemporaryDirectory() as tmp:
        shapes_file = os.path.join(tmp, "shapes.csv")
        write_shapes(cases, shapes_file)

        def worker(g: int) -> None:
            env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(g))
            for i, c in enumerate(cases):
                if i % ngpu != g:
                    continue
                tid = c["TestID"]
                cmd = [binary, "--shapes", shapes_file, "--only", tid, "--out", os.path.join(tmp, f"{tid}.csv"),
                       *extra]
                try:
                    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout_s)
                    msg = None if r.returncode == 0 else f"exit {r.returncode}: {r.stderr.strip()[-300:]}"
                except subprocess.TimeoutExpired:
                    msg = f"timed out after {timeout_s:.0f} s"
                if msg:
                    with lock:
                        failures.append(f"case {tid} (gpu {g}): {msg}")
                        print(f"case {tid} on gpu {g}: {msg}", file=log, flush=True)

        threads = [threading.Thread(target=worker, args=(g,)) for g in range(ngpu)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        parts = sorted(glob.glob(os.path.join(tmp, "*.csv")))
        parts = [p for p in parts if os.path.basename(p) != "shapes.csv"]
        n = merge_results(parts, out)
    print(f"wrote {out} ({n} rows) from {len(cases)} cases on {ngpu} GPU(s)", file=log, flush=True)
    return failures


def compare(paths: list[str], ours: str = "b200", other: str = "cublas_loop", worst: int = 8) -> dict:
    """Head-to-head of two backends over results CSVs (files, or directories of per-case CSVs)."""
    files: list[str] = []
    for p in paths:
        files += sorted(glob.glob(os.path.join(p, "*.csv"))) if os.path.isdir(p) else [p]
    by: dict[int, dict[str, dict]] = {}
    for p in files:
        with open(p, newline="") as f:
            for row in csv.DictReader(f):
                by.setdefault(int(row["TestID"]), {})[row["Backend"]] = row
    pairs = [(tid, d[ours], d[other]) for tid, d in sorted(by.items())
             if ours in d and other in d and d[ours]["Check"] == "PASS" and d[other]["Check"] in ("PASS", "SKIP")]
    not_ok = sorted(tid for tid, d in by.items() if any(r["Check"] not in ("PASS", "SKIP") for r in d.values()))
    n = len(pairs)
    rep = {"ours": ours, "other": other, "cases": n, "non_pass": not_ok}
    if n == 0:
        return rep
    t_ours = [float(a["Time_ms"]) for _, a, _ in pairs]
    t_other = [float(b["Time_ms"]) for _, _, b in pairs]
    f_ours = [float(a["TFLOPS"]) for _, a, _ in pairs]
    f_other = [float(b["TFLOPS"]) for _, _, b in pairs]
    rep.update(
        wins=sum(a > b for a, b in zip(f_ours, f_other)),
        geomean_speedup=math.exp(sum(math.log(b / a) for a, b in zip(t_ours, t_other)) / n),
        total_ms_ours=sum(t_ours), total_ms_other=sum(t_other),
        mean_tflops_ours=sum(f_ours) / n, mean_tflops_other=sum(f_other) / n,
        worst=[{"TestID": tid, "Case": a["Case"], "B": int(a["B"]), "M": int(a["M"]), "N": int(a["N"]),
                "K": int(a["K"]), "tflops_ours": float(a["TFLOPS"]), "tflops_other": float(b["TFLOPS"]),
                "ratio": float(a["TFLOPS"]) / float(b["TFLOPS"])}
               for tid, a, b in sorted(pairs, key=lambda t: float(t[1]["TFLOPS"]) / float(t[2]["TFLOPS"]))[:worst]],
    )
    return rep


def format_report(rep: dict) -> str:
    ours, other, n = rep["ours"], rep["other"], rep["cases"]
    lines = [f"{n} cases where {ours} PASSes and {other} PASSes or SKIPs; non-PASS cases: {rep['non_pass'][:10]}"]
    if n == 0:
        return "\n".join(lines)
    lines += [
        f"{ours} faster in {rep['wins']}/{n}",
        f"geomean speedup {ours} vs {other}: {rep['geomean_speedup']:.3f}x; total time {rep['total_ms_ours']:.1f} ms "
        f"vs {rep['total_ms_other']:.1f} ms ({rep['total_ms_other'] / rep['total_ms_ours']:.3f}x)",
        f"mean TFLOPS: {ours} {rep['mean_tflops_ours']:.0f}, {other} {rep['mean_tflops_other']:.0f}",
        f"worst cases for {ours} ({ours}/{other} TFLOPS):",
    ]
    for w in rep["worst"]:
        lines.append(f"  {w['TestID']:4d} {w['Case']:28s} B={w['B']:>3} M={w['M']:>5} N={w['N']:>5} K={w['K']:>5}  "
                     f"{w['tflops_ours']:6.0f} vs {w['tflops_other']:6.0f}  ({w['ratio']:.2f})")
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    extra: list[str] = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    ap = argparse.ArgumentParser(prog="suite.py")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="one gg_bench process per case over the GPUs")
    r.add_argument("shapes")
    r.add_argument("out")
    r.add_argument("--ngpu", type=int, default=1)
    r.add_argument("--timeout", type=float, default=300.0, help="seconds per case")
    c = sub.add_parser("compare", help="compare two backends over results CSVs")
    c.add_argument("paths", nargs="+")
    c.add_argument("--ours", default="b200")
    c.add_argument("--other", default="cublas_loop")
    a = ap.parse_args(argv)
    if a.cmd == "run":
        if a.ngpu < 1:
            ap.error("--ngpu must be >= 1")
        failures = run_suite(a.shapes, a.out, a.ngpu, a.timeout, extra)
        return 1 if failures else 0
    print(format_report(compare(a.paths, a.ours, a.other)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
