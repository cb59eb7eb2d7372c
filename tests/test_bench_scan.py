"""The scan benchmark in the reference's result format (mamba_ssm_benchmark_b200/bench_scan.py)."""

import csv
import json

import pytest
import torch

from conftest import load_golden
from mamba_ssm_benchmark_b200 import bench_scan


def test_inputs_match_reference_benchmark():
    """Same seeded inputs as benchmarks/bench_scan.py:make_inputs (recorded from the reference)."""
    want = load_golden("bench_inputs.npz")
    got = bench_scan.make_inputs(8, device="cpu")
    for name, t in zip(("x", "delta", "A", "Bm", "Cm"), got):
        assert torch.equal(t.detach(), want[name]), name
        assert t.requires_grad


def test_csv_has_reference_columns(tmp_path):
    res = {"env": {}, "config": dict(bench_scan.CONFIG),
           "runs": [{"scan": "b200", "L": 256, "fwd": {"ms": 0.1, "q25": 0.09, "q75": 0.11, "peak_mb": 1.0},
                     "fwd_bwd": {"oom": True}}]}
    path = tmp_path / "bench_scan.csv"
    bench_scan.write_csv(res, str(path))
    rows = list(csv.DictReader(open(path)))
    assert list(rows[0].keys()) == ["scan", "L", "fwd_ms", "fwd_q25", "fwd_q75", "fwd_peak_mb", "fwd_bwd_oom"]
    assert rows[0]["scan"] == "b200" and rows[0]["L"] == "256"


@pytest.mark.gpu
def test_benchmark_runs_and_writes_reference_layout(tmp_path):
    out, out_csv = tmp_path / "scan.json", tmp_path / "scan.csv"
    bench_scan.main(["--lengths", "256,1024", "--out", str(out), "--csv", str(out_csv)])
    res = json.load(open(out))
    assert res["config"] == {"B": 1, "D": 512, "N": 16}
    assert [r["L"] for r in res["runs"]] == [256, 1024]
    for r in res["runs"]:
        assert r["scan"] == "b200"
        for k in ("fwd", "fwd_bwd"):
            assert set(r[k]) == {"ms", "q25", "q75", "peak_mb"} and r[k]["ms"] > 0
    assert len(list(csv.DictReader(open(out_csv)))) == 2
