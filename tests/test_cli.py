"""The julia-cuda command-line front end (julia-cuda_b200/csrc/cli.cpp; the reference's src/main.rs
and src/serve.rs): argument handling on the CPU, and on the GPU the JSONL serving loop (one result
line per request, in order, the engine's logits), --check and --time."""
import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "julia-cuda_b200", "julia-cuda")


def run(args, stdin="", timeout=600):
    return subprocess.run([CLI] + args, input=stdin, capture_output=True, text=True,
                          timeout=timeout)


@pytest.fixture(scope="module")
def cli():
    if not os.path.exists(CLI):
        pytest.fail("julia-cuda_b200/julia-cuda is not built (make -C julia-cuda_b200)")
    return CLI


def test_usage_and_bad_arguments(cli):
    r = run(["--help"])
    assert r.returncode == 0 and "usage: julia-cuda" in r.stdout
    for bad in (["--bogus"], ["--mode"], ["--random", "1", "--set", "nope=3"],
                ["--random", "1", "--mode", "7"]):
        r = run(bad)
        assert r.returncode == 2, (bad, r.stderr)


def test_missing_model_directory_is_an_error(cli, tmp_path):
    r = run([str(tmp_path / "absent")])
    assert r.returncode == 1 and "julia-cuda:" in r.stderr


SMALL = ["--set", "d_model=256", "--set", "inter=256", "--set", "n_layers=3",
         "--set", "vocab=500", "--set", "head_ff=512", "--set", "scorer_hidden=128",
         "--set", "max_positions=512"]


@pytest.mark.gpu
def test_kernels_load_without_a_model(cli):
    r = run([])
    assert r.returncode == 0 and "load and run on" in r.stderr and "B200" in r.stderr


@pytest.mark.gpu
def test_serves_jsonl_like_the_engine(cli, jc):
    c = jc.default_config(d_model=256, inter=256, n_layers=3, vocab=500, head_ff=512,
                          scorer_hidden=128, max_positions=512)
    rng = np.random.default_rng(3)
    reqs, lines = [], []
    for i, n in enumerate([40, 293, 7, 511]):
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        mk = np.sort(rng.choice(n, min(4, n), replace=False)).astype(np.uint32)
        q = i % 3
        reqs.append((ids, mk, q))
        lines.append(json.dumps({"ids": ids.tolist(), "markers": mk.tolist(),
                                 "qtype": ["choice", "score", "noul"][q], "text": "ignored"}))
    r = run(["--random", "42", "--max-length", "512"] + SMALL, "\n".join(lines) + "\n")
    assert r.returncode == 0, r.stderr
    out = [json.loads(x) for x in r.stdout.splitlines()]
    assert len(out) == len(reqs) and "per request, GPU" in r.stderr
    eng = jc.Engine.load_random(c, 42, max_length=512)
    try:
        want, _ = eng.run(reqs)
    finally:
        eng.close()
    for o, w in zip(out, want):
        # Two runs of the same kernels differ only in the order of the row statistics' atomic
        # sums (a few ulps of the logits).
        got = np.asarray(o["logits"])
        assert np.max(np.abs(got - w)) < 1e-3
        p = np.exp(got - got.max())
        assert np.allclose(o["probabilities"], p / p.sum(), atol=1e-6)
        assert o["choice"] == int(np.argmax(got)) and o["gpu_ms"] > 0 and o["truncated"] is False


@pytest.mark.gpu
def test_bad_request_lines_are_reported(cli):
    r = run(["--random", "1", "--max-length", "128"] + SMALL,
            '{"ids": [1, 2, 3], "markers": [9]}\n')
    assert r.returncode == 1 and "line 1" in r.stderr
    r = run(["--random", "1", "--max-length", "128"] + SMALL, '{"markers": [0]}\n')
    assert r.returncode == 1 and "no \"ids\"" in r.stderr


@pytest.mark.gpu
def test_check_and_time(cli):
    r = run(["--random", "5", "--max-length", "512", "--check", "--time"] + SMALL)
    assert r.returncode == 0, r.stderr
    assert "check: ok" in r.stderr and "whole model, one persistent launch" in r.stderr
