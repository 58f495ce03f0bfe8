"""Requests packed into one forward (julia_cuda_set_packing): every request attends only to its
own tokens and restarts its RoPE positions, so its logits match running it alone (up to the
accumulation order of differently sized GEMM tiles and key tiles) and the oracle's f32 model (the
reference's bars: logits max |d| < 0.15, src/check.rs:560; mean |d| <= 0.03). Packs above 832
rows run the tcgen05 attention for the global layers, smaller ones the mma.sync kernel."""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def oracle_cfg(O, c):
    return O.Config(*[getattr(c, f) for f, _ in c._fields_])


@pytest.fixture(scope="module")
def packed_case(jc, O):
    rep = importlib.import_module("julia-cuda_b200.replicas")
    c = jc.default_config(max_positions=1024)
    raw = O.init_random(oracle_cfg(O, c), 99)
    eng = jc.Engine.load_raw(c, raw, max_length=1024)
    reqs = rep.serving_requests(10, 3, c.vocab)
    rng = np.random.default_rng(5)
    for n in (1, 63, 64, 65, 129):  # edge lengths: one token, one key tile, just past it
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        reqs.append((ids, np.unique(rng.integers(0, n, 2)).astype(np.uint32), 0))
    reqs = [(ids, mk, 1 if i % 5 == 4 else 0) for i, (ids, mk, _) in enumerate(reqs)]  # two types
    alone, _ = eng.run(reqs)
    eng.set_packing(1024)
    packed, ms = eng.run(reqs)
    yield c, raw, eng, reqs, alone, packed, ms
    eng.set_packing(0)
    eng.close()


def test_packed_requests_match_running_alone(jc, packed_case):
    c, raw, eng, reqs, alone, packed, ms = packed_case
    assert eng.device_error() == 0 and np.all(ms > 0)
    for a, p in zip(alone, packed):
        assert a.shape == p.shape
        assert np.max(np.abs(a - p)) < 2e-3


def test_packed_requests_match_the_f32_model(O, packed_case):
    c, raw, eng, reqs, alone, packed, ms = packed_case
    oc = oracle_cfg(O, c)
    d = []
    for (ids, mk, qt), p in zip(reqs, packed):
        want = O.forward_f32(oc, raw, ids, mk, qt)
        d.append(np.abs(p - want))
        assert np.argmax(p) == np.argmax(want) or np.sort(want)[-1] - np.sort(want)[-2] < 0.01
    d = np.concatenate(d)
    assert d.max() < 0.15 and d.mean() <= 0.03


def test_packs_share_their_time_and_persistent_modes_agree(jc, packed_case):
    c, raw, eng, reqs, alone, packed, ms = packed_case
    # Requests of one forward report the same time; there are fewer forwards than requests.
    assert len(set(np.round(ms, 6))) < len(reqs)
    for mode in (1, 2):
        out, _ = eng.run(reqs[:6], layer_fused=mode)
        for a, p in zip(alone[:6], out):
            assert np.max(np.abs(a - p)) < 2e-3, f"mode {mode}"


def test_packing_rejects_rows_above_max_length(jc, packed_case):
    c, raw, eng, reqs, alone, packed, ms = packed_case
    with pytest.raises(jc.JuliaCudaError):
        eng.set_packing(4096)


def test_large_packs_run_the_persistent_gemm(jc, O):
    """Packs of a few thousand rows: the GEMMs have more tiles than SMs (the persistent kernel,
    RoPE positions from each row's request), attention 64-query mma.sync CTAs bounded by each
    row's request. Each request's logits match running it alone."""
    rep = importlib.import_module("julia-cuda_b200.replicas")
    c = jc.default_config(max_positions=3072)
    eng = jc.Engine.load_raw(c, O.init_random(oracle_cfg(O, c), 7), max_length=3072)
    try:
        reqs = rep.serving_requests(24, 11, c.vocab)
        alone, _ = eng.run(reqs)
        eng.set_packing(3072)
        packed, ms = eng.run(reqs)
        assert eng.device_error() == 0 and len(set(np.round(ms, 6))) < len(reqs)
        for a, p in zip(alone, packed):
            assert np.max(np.abs(a - p)) < 2e-3
    finally:
        eng.close()
