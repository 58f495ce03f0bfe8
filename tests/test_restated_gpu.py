"""The reference's per-step GPU forward restated in CUDA C++ (baseline/restated), the latency
baseline of the headline: it must compute the same model before its time means anything. Its
logits are checked against the oracle's f32 model (the reference's bars: max |d| < 0.15,
src/check.rs:560; mean |d| <= 0.03) and against this library's engine, at lengths that take each
of the reference's three GEMM tile shapes (32, 64 and 128 rows: `gemm::choose`, src/gemm.rs:153-
166) and its split-K path (293 tokens: the 768-wide GEMMs fill less than half the SMs)."""
import ctypes
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline", "restated"))
import restated  # noqa: E402


def oracle_cfg(O, c):
    return O.Config(*[getattr(c, f) for f, _ in c._fields_])


def test_restated_library_exports_its_symbols():
    if not os.path.exists(restated.LIB_PATH):
        pytest.skip("baseline/restated is not built")
    L = ctypes.CDLL(restated.LIB_PATH)
    assert all(hasattr(L, s) for s in restated.SYMBOLS)


def test_restated_load_without_gpu_reports_an_error(jc):
    """No crash without a device (or with a bad raw size): NULL and a message."""
    if not os.path.exists(restated.LIB_PATH):
        pytest.skip("baseline/restated is not built")
    c = jc.default_config(max_positions=64)
    with pytest.raises(RuntimeError, match="restated"):
        restated.Restated(c, np.zeros(10, np.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [100, 293, 600])
def test_restated_forward_matches_the_model(jc, O, n):
    c = jc.default_config(max_positions=1024)
    raw = O.init_random(oracle_cfg(O, c), 4242)
    ref = restated.Restated(c, raw, max_length=1024)
    eng = jc.Engine.load_raw(c, raw, max_length=1024)
    try:
        rng = np.random.default_rng(n)
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
        for qtype in (0, 1):
            got, ms = ref.run(ids, markers, qtype)
            assert ms > 0
            want = O.forward_f32(oracle_cfg(O, c), raw, ids, markers, qtype)
            d = np.abs(got - want)
            assert d.max() < 0.15 and d.mean() <= 0.03, (n, qtype, d)
            ours, _ = eng.run([(ids, markers, qtype)])
            assert np.max(np.abs(ours[0] - got)) < 0.05
    finally:
        ref.close()
        eng.close()
