"""The tile plans against measured sweeps (the reference's plan_matches_the_sweeps,
src/forward.rs:815-823, for the B200), CPU only (the plans are host code):

- the per-step kernels' choice (jc_choose_gemm) must pick, for every encoder GEMM at BASELINE
  config 1's row counts on 148 SMs, a width whose measured time alone is within 5% of the fastest,
  and for packs of 2048-6144 rows a width and kernel (single-SM persistent, or CTA pairs where the
  default pair policy puts persistent 256-column launches) within 5% of the fastest of 128 and
  256 columns on either (tests/golden/gemm_tile_sweep.json, `python bench.py --tile-sweep` on a
  B200);
- the persistent kernel's plan (jc_persist_tile over jc_persist_phase_us) must give a whole
  persistent forward within 3% of the faster of its two forced widths at those row counts, in
  both persistent modes (tests/golden/persist_tile_sweep.json, `python bench.py --persist-sweep`),
  and the plan's own width choices must be the ones the sweep's planned runs used."""
import ctypes
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
SWEEP = os.path.join(HERE, "golden", "gemm_tile_sweep.json")
EPI = {"qkv": 20, "wo": 9, "wi": 6, "wo_mlp": 9}
SMS = 148


PERSIST = os.path.join(HERE, "golden", "persist_tile_sweep.json")


@pytest.fixture(scope="module")
def sweep():
    with open(SWEEP) as f:
        data = json.load(f)
    cases = {}
    for c in data["cases"]:
        cases.setdefault((c["gemm"], c["m"], c["n"], c["k"]), {})[(c["bn"], c.get("pair", False))] = c["us"]
    return cases


CONFIG_1 = (72, 293, 448, 1024)
PACKS = (2048, 3072, 6144)


def test_sweep_covers_config_1_and_packs(sweep):
    assert {(g, m) for g, m, _, _ in sweep} == {(g, m) for g in EPI for m in CONFIG_1 + PACKS}


@pytest.fixture(scope="module")
def persist_sweep():
    with open(PERSIST) as f:
        data = json.load(f)
    return {(c["mode"], c["m"], c["policy"]): c["us"] for c in data["cases"]}


def test_persistent_plan_matches_the_sweep(persist_sweep):
    """A planned persistent forward is within 3% of the faster forced width, in both modes."""
    for mode in (1, 2):
        for m in (72, 293, 448, 1024):
            t = {p: persist_sweep[(mode, m, p)] for p in (0, 32, 64)}
            assert t[0] <= 1.03 * min(t[32], t[64]), (mode, m, t)


def test_persistent_plan_is_the_swept_one(jc, sweep):
    """The plan behind the sweep's planned runs: RoPE and GeGLU phases at 64 columns, the
    768-wide phases at the width persist_phase_us prefers, which at these row counts is 64 (each
    item of a 32-column phase adds its report to the row block's completion)."""
    lib = jc.lib()
    for (g, m, n, k) in [c for c in sweep if c[1] in CONFIG_1]:
        assert lib.jc_persist_tile(m, n, k, EPI[g], SMS) == 64, (g, m)
        if g in ("wo", "wo_mlp"):
            assert lib.jc_persist_phase_us(m, n, k, 64, SMS) < lib.jc_persist_phase_us(m, n, k, 32, SMS)


def test_per_step_choice_matches_the_sweep(jc, sweep):
    """The per-step kernels' tile width (jc_choose_gemm; RoPE and GeGLU raise it to 64 columns)
    is within 5% of the fastest measured width; past one wave a 256-column launch runs on CTA
    pairs (the default pair policy)."""
    lib = jc.lib()
    for (g, m, n, k), us in sweep.items():
        bn, splits = ctypes.c_int(0), ctypes.c_int(0)
        lib.jc_choose_gemm(m, n, k, SMS, ctypes.byref(bn), ctypes.byref(splits))
        pick = max(bn.value, 64) if g in ("qkv", "wi") else bn.value
        persistent = pick >= 128 and -(-m // 128) * (n // pick) > SMS
        key = (pick, persistent and pick == 256)
        best = min(us.values())
        assert splits.value == 1 and us[key] <= 1.05 * best, (g, m, key, us)


def test_phase_cost_model(jc):
    """The model's terms: a tile costs its k-blocks' MMA chain and its width's epilogue; a phase
    pays one tile per wave of the grid."""
    lib = jc.lib()
    one = lib.jc_gemm_phase_us(293, 768, 768, 32, SMS)
    assert one == pytest.approx(0.8 + 0.163 * 12 + 0.70, rel=1e-9)
    assert lib.jc_gemm_phase_us(293, 768, 1152, 32, SMS) == pytest.approx(one + 0.163 * 6, rel=1e-9)
    # 1024 rows of 32-column tiles: 8 x 24 = 192 tiles, two waves on 148 CTAs
    assert lib.jc_gemm_phase_us(1024, 768, 768, 32, SMS) == pytest.approx(2 * one, rel=1e-9)
    assert lib.jc_gemm_phase_us(293, 768, 768, 48, SMS) == -1.0  # not a tile width
    assert lib.jc_gemm_phase_us(293, 800, 768, 64, SMS) == -1.0  # does not divide n
    # a persistent phase adds 0.19 us per item of a row block
    assert lib.jc_persist_phase_us(293, 768, 768, 32, SMS) == pytest.approx(one + 0.19 * 24, rel=1e-9)
    assert lib.jc_persist_phase_us(293, 768, 768, 128, SMS) == -1.0  # not a persistent width


def test_tile_policy_hook(jc):
    """jc_persist_tile_policy forces a width where the phase allows it and returns the old policy."""
    lib = jc.lib()
    assert jc.persist_tile_policy(32) == 0
    try:
        assert lib.jc_persist_tile(293, 768, 768, EPI["wo"], SMS) == 32
        assert lib.jc_persist_tile(293, 2304, 768, EPI["qkv"], SMS) == 64  # RoPE pairs span 64
        assert jc.persist_tile_policy(64) == 32
        assert lib.jc_persist_tile(293, 768, 768, EPI["wo"], SMS) == 64
        assert jc.persist_tile_policy(48) == -1  # refused: unchanged
        assert lib.jc_persist_tile(293, 768, 768, EPI["wo"], SMS) == 64
    finally:
        jc.persist_tile_policy(0)
    assert lib.jc_persist_tile(293, 768, 768, EPI["wo"], SMS) == 64
