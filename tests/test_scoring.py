"""The agreement scorer (the reference's tools/score.py checks, restated) on known cases."""
import importlib
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sc = importlib.import_module("julia-cuda_b200.scoring")


def test_agreement_counts_flips_and_deviations():
    want = [np.array([1.0, 0.0, -1.0]), np.array([0.0, 0.005]), np.array([2.0, -2.0])]
    got = [np.array([1.01, 0.0, -1.0]), np.array([0.006, 0.004]), np.array([-3.0, 2.0])]
    a = sc.agreement(got, want)
    assert a["requests"] == 3 and a["same_answer"] == 1
    assert abs(a["max_abs_dlogit"] - 5.0) < 1e-12
    assert abs(a["mean_abs_dlogit"] - (0.01 + 0.006 + 0.001 + 5.0 + 4.0) / 7) < 1e-12
    assert a["margin_hist"] == [1, 0, 0, 0, 0, 2]   # margins 0.005, 1.0 and 4.0 (bins [a, b))
    assert a["decided"] == 0                         # no margin above 2 x 5.0


def test_agreement_of_identical_runs():
    w = [np.arange(4.0), np.array([3.0, 1.0])]
    a = sc.agreement(w, w)
    assert a["agreement"] == 1.0 and a["max_abs_dlogit"] == 0.0 and a["decided_agreement"] == 1.0


def test_score_files_matches_the_reference_line(tmp_path):
    labels = [{"keys": ["a", "b", "c"], "gold": "b"}, {"keys": ["x", "y"], "gold": "x"}]
    res = [{"logits": [0.1, 0.9, 0.0]}, {"logits": [0.2, 0.7]}]
    base = [{"logits": [0.1, 0.8, 0.0]}, {"logits": [0.9, 0.1]}]
    for name, rows in (("labels", labels), ("res", res), ("base", base)):
        with open(tmp_path / f"{name}.jsonl", "w") as f:
            f.write("\n".join(json.dumps(r) for r in rows) + "\n")
    out = subprocess.run([sys.executable, "-m", "julia-cuda_b200.scoring", str(tmp_path / "labels.jsonl"),
                          str(tmp_path / "res.jsonl"), str(tmp_path / "base.jsonl")],
                         cwd=ROOT, capture_output=True, text=True, check=True).stdout
    assert "1/2 correct" in out and "same answer as baseline 1/2" in out
    assert "mean |dlogit| 0.2800" in out and "max 0.700" in out
