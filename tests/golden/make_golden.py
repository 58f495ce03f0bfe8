"""Regenerates the committed golden fixtures in this directory.

reference_known_answers.json: the literal expected values of the reference's own pure unit tests
(arnu515/julia-cuda, which has no shipped numeric fixtures: every checkpoint-based test skips
without the model):
  - src/forward.rs:815-823 `plan_matches_the_sweeps`: gemm_plan picks on 68 SMs x 2 blocks;
  - src/prep.rs:278-314 `bias_fold_matches_layernorm_then_linear`: xorshift seed, sizes, tolerance;
  - src/prep.rs:252-274 / :318-327: the permutation tests' sizes.

oracle_small.npz: a seeded small model run through the C oracle (f32 model and f16 emulation) and
through the independent torch restatement (tests/torch_ref.py), which must agree when generated.

Run: python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as O  # noqa: E402
import torch_ref  # noqa: E402


def small_config():
    return O.config(d_model=128, inter=128, n_layers=4, vocab=500, head_ff=256, scorer_hidden=128,
                    window=8, max_positions=256)


def main():
    known = {
        "plan_matches_the_sweeps": {
            "source": "src/forward.rs:815-823",
            "inter": 1152, "d_model": 384, "sms": 68, "per_sm": 2,
            "shapes": [[3 * 384, 384], [384, 384], [2 * 1152, 384], [384, 1152]],
            "picks": {"72": [[32, 1], [32, 3], [32, 1], [32, 3]],
                      "363": [[64, 1], [32, 1], [64, 1], [64, 3]],
                      "512": [[64, 1], [32, 1], [64, 1], [32, 1]]},
        },
        "bias_fold_matches_layernorm_then_linear": {
            "source": "src/prep.rs:278-314",
            "seed": "0x9e3779b97f4a7c15", "k": 64, "out": 32, "rows": 5, "row_offset": 3.0,
            "ln_eps": 1e-5, "tolerance": 2e-2,
        },
        "interleave_matches_the_geglu_epilogue": {"source": "src/prep.rs:252-274", "n": 2304,
                                                  "inter": 1152},
        "rope_permutation_pairs_rotate_half_dims": {"source": "src/prep.rs:318-327",
                                                    "n": 3 * 384},
    }
    with open(os.path.join(HERE, "reference_known_answers.json"), "w") as f:
        json.dump(known, f, indent=1)

    c = small_config()
    raw = O.init_random(c, 7)
    rng = np.random.default_rng(11)
    n = 40
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.array([0, 9, 23, 39], np.uint32)
    f32, tr32 = O.forward_f32(c, raw, ids, markers, 1, trace=True)
    emu, tr_emu = O.forward_emu(c, raw, ids, markers, 1, trace=True)
    tor, tr_t = torch_ref.forward(c, raw, ids, markers, 1, trace=True)
    assert np.max(np.abs(f32 - tor)) < 1e-4, (f32, tor)
    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), seed=7, ids=ids, markers=markers,
                        qtype=1, logits_f32=f32, logits_emu=emu, logits_torch=tor,
                        trace_f32=tr32.astype(np.float32))
    print("logits f32", f32, "emu", emu, "torch", tor)


if __name__ == "__main__":
    main()
