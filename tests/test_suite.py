"""The suite workflow (groupgemm-cktile-optimized_b200/suite.py): the one-process-per-case runner
(the reference's scripts/run_parallel.sh) and the two-backend comparison report
(scripts/compare.py). CPU tests drive the runner with a stand-in harness and check the report on
a hand-made results CSV; the GPU test runs the real harness with all three backends (b200 and
the two cuBLAS baselines) and requires every row to PASS the sampled fp32 check."""
import csv
import importlib.util
import math
import os
import stat
import sys

import pytest

from conftest import PKG_DIR, ROOT

HEADER = "TestID,Case,B,M,N,K,Dtype,GPU,Backend,Check,Time_ms,TFLOPS,MaxAbsErr,Detail,PctDensePeak"


def _suite():
    spec = importlib.util.spec_from_file_location("gg_suite", os.path.join(PKG_DIR, "suite.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _row(tid, case, backend, check, ms, tflops):
    return f'{tid},{case},2,64,128,256,bf16,"GPU",{backend},{check},{ms},{tflops},0.1,"d",1.0'


def test_compare_report_on_a_hand_made_csv(tmp_path):
    suite = _suite()
    p = tmp_path / "r.csv"
    p.write_text("\n".join([
        HEADER,
        _row(1, "A", "b200", "PASS", 1.0, 200.0), _row(1, "A", "cublas_loop", "PASS", 2.0, 100.0),
        _row(2, "B", "b200", "PASS", 4.0, 50.0), _row(2, "B", "cublas_loop", "PASS", 2.0, 100.0),
        _row(3, "C", "b200", "PASS", 1.0, 300.0), _row(3, "C", "cublas_loop", "SKIP", 3.0, 100.0),
        _row(4, "D", "b200", "FAIL", 1.0, 300.0), _row(4, "D", "cublas_loop", "PASS", 3.0, 100.0),
        _row(5, "E", "b200", "PASS", 1.0, 300.0),  # no partner row: not a pair
    ]) + "\n")
    rep = suite.compare([str(p)])
    assert rep["cases"] == 3 and rep["wins"] == 2 and rep["non_pass"] == [4]
    assert math.isclose(rep["geomean_speedup"], (2.0 * 0.5 * 3.0) ** (1 / 3))
    assert rep["total_ms_ours"] == 6.0 and rep["total_ms_other"] == 7.0
    assert math.isclose(rep["mean_tflops_ours"], 550.0 / 3) and math.isclose(rep["mean_tflops_other"], 100.0)
    assert [w["TestID"] for w in rep["worst"]] == [2, 1, 3]
    assert rep["worst"][0]["ratio"] == 0.5
    text = suite.format_report(rep)
    assert "b200 faster in 2/3" in text and "1.442x" in text and "non-PASS cases: [4]" in text
    # a directory of per-case files reads the same as the merged file
    d = tmp_path / "cases"
    d.mkdir()
    lines = p.read_text().splitlines()
    for tid in range(1, 6):
        (d / f"{tid}.csv").write_text("\n".join([HEADER] + [l for l in lines[1:] if l.startswith(f"{tid},")]) + "\n")
    assert suite.compare([str(d)]) == rep


def test_compare_with_no_common_case(tmp_path):
    suite = _suite()
    p = tmp_path / "r.csv"
    p.write_text(HEADER + "\n" + _row(1, "A", "b200", "PASS", 1.0, 1.0) + "\n")
    rep = suite.compare([str(p)], other="cublas_grouped")
    assert rep["cases"] == 0 and "0 cases" in suite.format_report(rep)


FAKE = r'''#!{python}
# Stand-in for gg_bench: writes a one-case results CSV for --only ID; case 3 fails, case 4 hangs.
import os, sys, time
a = sys.argv[1:]
shapes, only, out = a[a.index("--shapes") + 1], a[a.index("--only") + 1], a[a.index("--out") + 1]
rows = [l.strip().split(",") for l in open(shapes)][1:]
row = [r for r in rows if r[0] == only][0]
if only == "3":
    sys.exit(1)
if only == "4":
    time.sleep(30)
with open(out, "w") as f:
    f.write("{header}\n")
    for b in ("b200", "cublas_loop"):
        f.write(",".join(row + ["bf16", "gpu" + os.environ["CUDA_VISIBLE_DEVICES"], b, "PASS", "1.0", "1.0", "0", "x",
                                " ".join(a[a.index("--out") + 2:]) or "-"]) + "\n")
'''


def test_runner_one_process_per_case_over_gpus(tmp_path):
    suite = _suite()
    fake = tmp_path / "fake_bench"
    fake.write_text(FAKE.format(python=sys.executable, header=HEADER))
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    shapes = tmp_path / "shapes.csv"
    # a results file as shapes: duplicate TestIDs (one row per backend) are one case
    shapes.write_text("\n".join([HEADER] + [_row(t, f"C{t}", b, "PASS", 1, 1) for t in (5, 1, 2, 3, 4, 6)
                                            for b in ("b200", "cublas_loop")]) + "\n")
    assert [c["TestID"] for c in suite.read_shapes(str(shapes))] == ["5", "1", "2", "3", "4", "6"]
    out = tmp_path / "out.csv"
    failures = suite.run_suite(str(shapes), str(out), ngpu=2, timeout_s=3, extra=["--iters", "2"],
                               binary=str(fake), log=open(os.devnull, "w"))
    assert sorted(f.split()[1] for f in failures) == ["3", "4"]
    assert any("timed out" in f for f in failures)
    rows = list(csv.DictReader(open(out)))
    assert [r["TestID"] for r in rows] == ["1", "1", "2", "2", "5", "5", "6", "6"]
    # round-robin over the two GPUs in file order: 5 -> gpu0, 1 -> gpu1, 2 -> gpu0, 6 -> gpu1
    gpu = {r["TestID"]: r["GPU"] for r in rows}
    assert gpu == {"1": "gpu1", "2": "gpu0", "5": "gpu0", "6": "gpu1"}
    assert all(r["PctDensePeak"] == "--iters 2" for r in rows)  # extra args reach the harness


def test_cli_compare_prints_report(tmp_path, capsys):
    suite = _suite()
    p = tmp_path / "r.csv"
    p.write_text("\n".join([HEADER, _row(1, "A", "b200", "PASS", 1.0, 200.0),
                            _row(1, "A", "cublas_loop", "PASS", 2.0, 100.0)]) + "\n")
    assert suite.main(["compare", str(p)]) == 0
    assert "b200 faster in 1/1" in capsys.readouterr().out


def test_committed_suite_results_reproduce_the_summary():
    """The 360-case results file under profiles/ gives the figures its summary quotes."""
    suite = _suite()
    path = os.path.join(ROOT, "profiles", "full_suite_360_b200_vs_cublas.csv")
    rep = suite.compare([path])
    assert rep["cases"] == 360 and rep["non_pass"] == []
    summary = open(os.path.join(ROOT, "profiles", "full_suite_360_b200_vs_cublas.md")).read()
    assert f"{rep['geomean_speedup']:.3f}x" in summary
    assert f"{rep['wins']}/360" in summary


@pytest.mark.gpu
@pytest.mark.parametrize("shapes,only", [("pad.csv", None), ("baseline.csv", "1001")])
def test_runner_all_backends_pass_the_check(tmp_path, shapes, only):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    suite = _suite()
    src = os.path.join(PKG_DIR, "shapes", shapes)
    if only:
        cases = [c for c in suite.read_shapes(src) if c["TestID"] == only]
        src = str(tmp_path / "shapes.csv")
        suite.write_shapes(cases, src)
    out = tmp_path / "results.csv"
    failures = suite.run_suite(src, str(out), ngpu=1, timeout_s=300,
                               extra=["--backends", "b200,cublas_loop,cublas_grouped", "--warmup", "2", "--iters", "3"])
    assert failures == []
    rows = list(csv.DictReader(open(out)))
    n_cases = len(suite.read_shapes(src))
    assert len(rows) == 3 * n_cases
    for row in rows:
        assert row["Check"] == "PASS", row
        assert float(row["TFLOPS"]) > 0
    assert {r["Backend"] for r in rows} == {"b200", "cublas_loop", "cublas_grouped"}
    rep = suite.compare([str(out)], other="cublas_grouped")
    assert rep["cases"] == n_cases and rep["non_pass"] == []
