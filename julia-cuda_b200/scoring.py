"""Agreement between two runs' logits, and accuracy against labels: the checks of the reference's
tools/score.py (accuracy of the argmax answer against `gold`; against a baseline run, how many
answers are the same and the mean / max |delta logit|), plus the margin histogram north_star's
parity gate asks for.

    python -m julia-cuda_b200.scoring labels.jsonl results.jsonl [baseline.jsonl]

reads the reference's formats: a results line holds `logits` (one per marker) and optionally
`probabilities`; a labels line holds `keys` (one per marker) and `gold` (the right key).
"""
from __future__ import annotations

import json
import sys

import numpy as np

MARGIN_BINS = (0.0, 0.01, 0.03, 0.1, 0.3, 1.0, np.inf)


def agreement(got, want) -> dict:
    """got, want: sequences of per-request logit vectors (want the baseline). Returns the
    requests, how many pick the same argmax, mean and max |delta logit| over all markers, the
    histogram of the baseline's top-2 margins (bins MARGIN_BINS), and the agreement among the
    requests whose baseline margin exceeds twice the largest deviation (a flip there is an
    error, not a near tie)."""
    got = [np.asarray(g, np.float64) for g in got]
    want = [np.asarray(w, np.float64) for w in want]
    if len(got) != len(want) or any(g.shape != w.shape for g, w in zip(got, want)):
        raise ValueError("agreement: runs of different shapes")
    d = np.concatenate([np.abs(g - w) for g, w in zip(got, want)]) if got else np.zeros(0)
    same = np.array([g.size > 0 and np.argmax(g) == np.argmax(w) for g, w in zip(got, want)])
    margins = np.array([np.sort(w)[-1] - np.sort(w)[-2] if w.size > 1 else np.inf for w in want])
    max_d = float(d.max()) if d.size else 0.0
    decided = margins > 2 * max_d
    return {
        "requests": len(got),
        "same_answer": int(same.sum()),
        "agreement": float(same.mean()) if len(got) else 1.0,
        "mean_abs_dlogit": float(d.mean()) if d.size else 0.0,
        "max_abs_dlogit": max_d,
        "margin_hist": np.histogram(margins, bins=MARGIN_BINS)[0].tolist(),
        "decided": int(decided.sum()),
        "decided_agreement": float(same[decided].mean()) if decided.any() else 1.0,
    }


def accuracy(results, labels) -> tuple[int, int]:
    """(correct, total): the argmax marker's key against `gold`, per request."""
    correct = 0
    for r, lab in zip(results, labels):
        scores = r.get("probabilities", r.get("logits"))
        pick = int(np.argmax(scores))
        correct += int(lab["keys"][pick] == lab["gold"])
    return correct, len(labels)


def _read(path):
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def score_files(labels_path: str, results_path: str, baseline_path: str | None = None) -> str:
    """The reference script's line: accuracy, and agreement with a baseline run if given."""
    labels, res = _read(labels_path), _read(results_path)
    correct, total = accuracy(res, labels)
    line = f"{results_path}: {correct}/{total} correct"
    if baseline_path:
        base = _read(baseline_path)
        a = agreement([r["logits"] for r in res], [b["logits"] for b in base])
        line += (f" | same answer as baseline {a['same_answer']}/{a['requests']} | mean |dlogit| "
                 f"{a['mean_abs_dlogit']:.4f} max {a['max_abs_dlogit']:.3f} | baseline top-2 "
                 f"margins <0.01/<0.03/<0.1/<0.3/<1/>=1: {a['margin_hist']}")
    return line


if __name__ == "__main__":
    if len(sys.argv) not in (3, 4):
        sys.exit(__doc__)
    print(score_files(*sys.argv[1:]))
