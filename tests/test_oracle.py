"""The CPU oracle against the reference's own known-answer tests, an independent torch restatement,
the committed fixtures, and the reference's tolerance design. CPU only."""
import json
import os

import numpy as np
import pytest

import torch_ref

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def known():
    with open(os.path.join(GOLDEN, "reference_known_answers.json")) as f:
        return json.load(f)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ---- the reference's pure tests, restated ----

def test_reference_interleave_known_answer(O):
    """src/prep.rs:252-274: the reference's GeGLU row order against its epilogue's fragment map."""
    k = known()["interleave_matches_the_geglu_epilogue"]
    n, inter = k["n"], k["inter"]
    rows = O.ref_interleave_geglu_rows(n)
    seen = np.zeros(inter, bool)
    for bx in range(n // 64):
        for wc in range(2):
            for lane in range(32):
                e0 = (lane & 3) * 2
                cw = 64 * bx + 32 * wc + e0
                for q in range(2):
                    for e in range(2):
                        col = 32 * bx + 16 * wc + e0 + 8 * q + e
                        assert rows[cw + 16 * q + e] == col
                        assert rows[cw + 16 * q + 8 + e] == inter + col
                        seen[col] = True
    assert seen.all()


def test_reference_rope_permutation_known_answer(O):
    """src/prep.rs:318-327."""
    n = known()["rope_permutation_pairs_rotate_half_dims"]["n"]
    rows = O.ref_permute_rope_rows(n)
    for p in range(0, 2 * n // 3, 2):
        head, i = p // 64, (p % 64) // 2
        assert (rows[p], rows[p + 1]) == (64 * head + i, 64 * head + i + 32)
    assert all(rows[p] == p for p in range(2 * n // 3, n))


def xorshift_stream(seed):
    """The reference test's generator (src/prep.rs:281-287)."""
    s = seed
    M = (1 << 64) - 1
    while True:
        s ^= (s << 13) & M
        s ^= s >> 7
        s ^= (s << 17) & M
        yield np.float32((s >> 40) / float(1 << 24) - 0.5)


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_bias_fold_known_answer(O, jc, impl):
    """src/prep.rs:278-314: the LayerNorm (with bias) fold against LN then linear in f64."""
    k = known()["bias_fold_matches_layernorm_then_linear"]
    K, out, rows = k["k"], k["out"], k["rows"]
    g = xorshift_stream(int(k["seed"], 16))
    w = np.array([next(g) for _ in range(out * K)], np.float32).reshape(out, K)
    gb = [(np.float32(1.0) + next(g), next(g)) for _ in range(K)]
    gamma = np.array([a for a, _ in gb], np.float32)
    beta = np.array([b for _, b in gb], np.float32)
    b = np.array([next(g) for _ in range(out)], np.float32)
    x = np.array([np.float32(k["row_offset"]) + next(g) for _ in range(rows * K)],
                 np.float32).reshape(rows, K)
    if impl == "oracle":
        w16, cs, bias = O.fold_layernorm_bias(w, gamma, beta, b)
    else:
        w16, cs, bias = jc.prep_fold_layernorm_bias(w, gamma, beta, b)
    wf = w16.view(np.float16).astype(np.float64)
    for row in x.astype(np.float64):
        mean = row.mean()
        r = 1 / np.sqrt(((row - mean) ** 2).mean() + k["ln_eps"])
        ln = (row - mean) * r * gamma + beta
        want = w.astype(np.float64) @ ln + b
        acc = wf @ row
        got = r * (acc - mean * cs.astype(np.float64)) + bias
        assert np.max(np.abs(got - want)) < k["tolerance"]


def test_plan_matches_the_sweeps(O):
    """src/forward.rs:815-823: the reference's layer-kernel plan model on a 2080 Ti."""
    k = known()["plan_matches_the_sweeps"]
    for n, picks in k["picks"].items():
        got = [list(O.ref_gemm_plan(int(n), cols, kk, k["sms"], k["per_sm"]))
               for cols, kk in k["shapes"]]
        assert got == picks, (n, got)


# ---- the oracle's model against an independent restatement and the fixtures ----

def small(O, **kw):
    base = dict(d_model=128, inter=128, n_layers=4, vocab=500, head_ff=256, scorer_hidden=128,
                window=8, max_positions=256)
    base.update(kw)
    return O.config(**base)


@pytest.mark.parametrize("n,window,qtype", [(1, 8, 0), (17, 8, 2), (70, 8, 1), (70, 0, 0)])
def test_oracle_f32_matches_torch(O, n, window, qtype):
    c = small(O, window=window)
    raw = O.init_random(c, 3)
    rng = np.random.default_rng(n)
    ids = rng.integers(0, c.vocab, n)
    markers = sorted(set(rng.integers(0, n, 3).tolist()))
    got, tr = O.forward_f32(c, raw, ids, markers, qtype, trace=True)
    want, trw = torch_ref.forward(c, raw, ids, markers, qtype, trace=True)
    assert np.max(np.abs(got - want)) < 2e-5
    for l in range(c.n_layers):
        assert rel_err(tr[l], trw[l]) < 1e-5


@pytest.mark.parametrize("n,head_rows", [(70, 40), (70, 70), (70, 200)])
def test_oracle_head_rows_matches_torch(O, n, head_rows):
    """The head limited to the first head_rows rows: the oracle's f32 path
    against the torch restatement, the emulation within the f16 bar, and markers past the head's
    rows rejected."""
    c = small(O)
    raw = O.init_random(c, 4)
    rng = np.random.default_rng(n + head_rows)
    ids = rng.integers(0, c.vocab, n)
    markers = [0, 17, min(n, head_rows) - 1]
    got = O.forward_f32(c, raw, ids, markers, 1, head_rows=head_rows)
    want = torch_ref.forward(c, raw, ids, markers, 1, head_rows=head_rows)
    assert np.max(np.abs(got - want)) < 2e-5
    emu = O.forward_emu(c, raw, ids, markers, 1, head_rows=head_rows)
    assert np.max(np.abs(emu - got)) < 3e-2
    if head_rows >= n:
        assert np.array_equal(got, O.forward_f32(c, raw, ids, markers, 1))
    else:
        assert np.max(np.abs(got - O.forward_f32(c, raw, ids, markers, 1))) > 1e-6
        with pytest.raises(ValueError):
            O.forward_f32(c, raw, ids, [head_rows], 1, head_rows=head_rows)
        with pytest.raises(ValueError):
            O.forward_emu(c, raw, ids, [head_rows], 1, head_rows=head_rows)


def test_oracle_reference_width(O):
    """The reference's own width (384 / 6 heads, scorer D -> D), torch vs oracle."""
    c = O.reference_width_config(n_layers=2, vocab=300, head_ff=256, max_positions=128)
    raw = O.init_random(c, 5)
    ids = np.arange(50) * 5 % c.vocab
    got = O.forward_f32(c, raw, ids, [1, 30, 49], 0)
    want = torch_ref.forward(c, raw, ids, [1, 30, 49], 0)
    assert np.max(np.abs(got - want)) < 2e-5


def test_golden_fixture(O):
    g = np.load(os.path.join(GOLDEN, "oracle_small.npz"))
    c = small(O)
    raw = O.init_random(c, int(g["seed"]))
    f32, tr = O.forward_f32(c, raw, g["ids"], g["markers"], int(g["qtype"]), trace=True)
    emu = O.forward_emu(c, raw, g["ids"], g["markers"], int(g["qtype"]))
    assert np.max(np.abs(f32 - g["logits_f32"])) < 1e-6
    assert np.max(np.abs(f32 - g["logits_torch"])) < 1e-4
    assert np.max(np.abs(emu - g["logits_emu"])) < 1e-6
    assert rel_err(tr, g["trace_f32"]) < 1e-6


def test_emulation_within_reference_tolerances(O):
    """The f16 emulation (what a correct kernel computes) against the f32 model, with the
    reference's chained limit (src/check.rs:395-402) and logit limits (:560, README.md:34)."""
    c = small(O, n_layers=6)
    raw = O.init_random(c, 9)
    rng = np.random.default_rng(0)
    ids = rng.integers(0, c.vocab, 120)
    markers = [0, 50, 99, 119]
    f32, t32 = O.forward_f32(c, raw, ids, markers, 0, trace=True)
    emu, temu = O.forward_emu(c, raw, ids, markers, 0, trace=True)
    for l in range(c.n_layers):
        assert rel_err(temu[l], t32[l]) < 3e-2
    assert np.max(np.abs(emu - f32)) < 0.15
    assert np.mean(np.abs(emu - f32)) <= 0.03


# ---- single-kernel emulation and the reference's negative tests (src/check.rs:1132-1184) ----

def test_negative_no_rope_fails(O):
    n, D = 64, 128
    a = O.f16(O.normal((n, D), 1))
    w = O.f16(O.normal((3 * D, D), 2, std=0.05))
    rope = O.rope_table(10000.0, n)
    with_rope, _ = O.emu_gemm(O.OR_ROPE, a, w, n, 3 * D, D, rope=rope)
    without, _ = O.emu_gemm(0, a, w, n, 3 * D, D)
    assert rel_err(O.f32(without), O.f32(with_rope)) > 3e-2


def test_negative_geglu_order_fails(O):
    n, D, I = 32, 128, 128
    a = O.f16(O.normal((n, D), 3))
    w = O.f16(O.normal((2 * I, D), 4, std=0.05))
    stats = O.row_stats(a)
    gamma = np.ones(D, np.float32)
    cs = O.f32(w).astype(np.float64).sum(1).astype(np.float32)
    good, _ = O.emu_gemm(O.OR_LN | O.OR_GEGLU, a, w, n, 2 * I, D, stats_in=stats, colsum=cs)
    swapped_w = np.concatenate([w[I:], w[:I]])
    swapped_cs = np.concatenate([cs[I:], cs[:I]])
    bad, _ = O.emu_gemm(O.OR_LN | O.OR_GEGLU, a, swapped_w, n, 2 * I, D, stats_in=stats,
                        colsum=swapped_cs)
    assert rel_err(O.f32(bad), O.f32(good)) > 3e-2


def test_negative_no_window_fails(O):
    n, H = 200, 2
    qkv = O.f16(O.normal((n, 3 * H * 64), 5))
    win = O.emu_attention(qkv, n, H, 64)
    glob = O.emu_attention(qkv, n, H, 0)
    assert rel_err(O.f32(glob), O.f32(win)) > 4e-3


def test_emu_attention_close_to_f32(O):
    """P rounded to f16 costs little (the reference's attention limit 4e-3, src/check.rs:384)."""
    n, H = 150, 2
    qkv = O.normal((n, 3 * H * 64), 6)
    q16 = O.f16(qkv)
    for window in (0, 64):
        e = O.f32(O.emu_attention(q16, n, H, window))
        f = O.attention_f32(O.f32(q16), n, H, window)
        assert rel_err(e, f) < 4e-3
