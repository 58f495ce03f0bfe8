"""Regenerates tests/golden/agreement_f32.npz: the f32 model's logits (the oracle, oracle/oracle.c,
restating julia-rs's forward as the reference's src/check.rs:177-224 and :484-548 call it) for the
argmax-agreement gate's request set, so the GPU test compares 1000 requests without spending
minutes of the GPU box's host time on the f32 model.

The set is BASELINE config 3's distribution, seeded: 1000 requests with log-normal lengths (mean
293, sigma 0.5, clipped to [32, 1024]; julia-cuda_b200/replicas.py serving_requests, seed
SEED), 4 markers each, question types cycling 0, 1, 2, through the benchmark model (hidden 768,
22 layers, head, scorer; seeded random weights, MODEL_SEED). The file keeps each request's
length, markers, question type and a checksum of its token ids (the test regenerates the ids
from the seed and checks them against it), and the f32 logits.

Run: python tests/golden/make_agreement.py   (about 10 minutes on 8 host threads)
"""
import importlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

COUNT = 1000
SEED = 2026
MODEL_SEED = 1234
OUT = os.path.join(HERE, "agreement_f32.npz")


def requests():
    """The gate's request set: (ids, markers, qtype) per request."""
    rep = importlib.import_module("julia-cuda_b200.replicas")
    reqs = rep.serving_requests(COUNT, SEED, 50368)
    return [(ids, mk, i % 3) for i, (ids, mk, _) in enumerate(reqs)]


def ids_checksum(ids) -> int:
    ids = np.asarray(ids, np.int64)
    return int((ids * (np.arange(len(ids), dtype=np.int64) % 997 + 1)).sum())


def main():
    c = O.config(max_positions=1024)
    raw = O.init_random(c, MODEL_SEED)
    reqs = requests()
    t0 = time.time()
    logits = np.zeros((COUNT, 4), np.float32)
    for i, (ids, mk, q) in enumerate(reqs):
        logits[i] = O.forward_f32(c, raw, ids, mk, q)
        if i % 100 == 99:
            print(f"{i + 1} requests, {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(
        OUT, count=COUNT, seed=SEED, model_seed=MODEL_SEED,
        lengths=np.array([len(r[0]) for r in reqs], np.int32),
        markers=np.stack([r[1] for r in reqs]).astype(np.uint32),
        qtypes=np.array([r[2] for r in reqs], np.int32),
        ids_checksum=np.array([ids_checksum(r[0]) for r in reqs], np.int64),
        logits=logits)
    print(f"wrote {OUT} ({time.time() - t0:.0f} s)")


if __name__ == "__main__":
    main()
