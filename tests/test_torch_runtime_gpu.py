"""This library against the torch runtime on the same checkpoint and GPU, as the reference compares
its engine with the original PyTorch runtime (tools/torch_baseline.py, then tools/score.py): the
runtime here is baseline/torch_runtime.py (transformers' ModernBertModel for the encoder, torch's
TransformerEncoderLayer head and LayerNorm / Linear / GELU scorer; pinned to the oracle by
tests/test_hf_modernbert.py), in f32. 48 seeded config-3 requests (log-normal lengths, 4 markers,
question types 0/1/2) through julia_cuda_run. Asserted: the same answer for every request whose
torch top-2 margin exceeds twice the largest deviation, and the largest |delta logit| within 3% of
the logits' rms (the parity gate's bar against the oracle)."""
import importlib
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytest.importorskip("transformers")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_engine_agrees_with_the_torch_runtime(jc, tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from torch_runtime import TorchRuntime
    replicas = importlib.import_module("julia-cuda_b200.replicas")
    scoring = importlib.import_module("julia-cuda_b200.scoring")
    cfg = jc.default_config(max_positions=1024)
    jc.save_checkpoint(str(tmp_path), cfg, jc.init_random(cfg, 77))
    eng = jc.Engine.load(str(tmp_path), max_length=1024)
    rt = TorchRuntime(str(tmp_path), device="cuda", dtype="fp32")
    reqs = [(ids, mk, i % 3) for i, (ids, mk, _) in
            enumerate(replicas.serving_requests(48, 78, cfg.vocab))]
    try:
        ours = [eng.run([r])[0][0] for r in reqs]
    finally:
        eng.close()
    theirs = [rt.forward(*r) for r in reqs]
    a = scoring.agreement(ours, theirs)
    rms = float(np.sqrt(np.mean(np.concatenate(theirs).astype(np.float64) ** 2)))
    print(f"agreement {a['same_answer']}/{a['requests']}, decided {a['decided']}, max |dlogit| "
          f"{a['max_abs_dlogit']:.2e} = {a['max_abs_dlogit'] / rms:.2%} of rms, mean "
          f"{a['mean_abs_dlogit']:.2e}")
    assert a["decided_agreement"] == 1.0, a
    assert a["max_abs_dlogit"] / rms < 0.03, a
