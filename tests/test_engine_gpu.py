"""The whole forward pass on the GPU (embed -> encoder -> head -> scorer), through the engine's C ABI,
against the oracle: the f16 emulation of the same arithmetic (tight) and the f32 model (the
reference's bars: chained stream within 3e-2, src/check.rs:395-402; logits max |d| < 0.15,
src/check.rs:560; mean |d| <= 0.03 and the same argmax).

Random-init logits are a few hundredths, so the absolute logit bars alone would pass a scorer
that outputs zeros: every logit check here is also relative to the logits' own scale
(rel_logits: max |d| / rms of the reference logits), and the head and the scorer are traced stage
by stage (julia_cuda_forward_trace) and bounded like the encoder's layers, as the reference's
--check bounds the head from the encoder output (src/check.rs:564-596). A planted mistake in the
oracle (a head bias left out) must fail these bars."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def rel_logits(got, want):
    """max |got - want| over the scale of `want` (its rms)."""
    w = np.asarray(want, np.float64)
    d = np.abs(np.asarray(got, np.float64) - w)
    return float(d.max() / max(float(np.sqrt(np.mean(w * w))), 1e-30))


# Bars relative to the logits' scale: against the f16 emulation (the same arithmetic; only the
# order of f32 sums and atomics differs) and against the f32 model.
LOGIT_REL_EMU = 1e-2
LOGIT_REL_F32 = 2e-2
# Per traced stage (encoder layer, head stage, scorer hidden layer), Frobenius-relative: against
# the emulation at four layers (TRACE_EMU) and over the whole 22-layer chain (TRACE_EMU_CHAIN),
# and against the f32 model (a third of the reference's chained bar, src/check.rs:395-402).
# Measured on a B200: 1e-4 to 4e-4 (small model), 1.1e-3 to 1.9e-3 (22 layers), logits 2e-3 of
# their scale against both references; the planted mistake moves the logits by 2.5e-2.
TRACE_EMU = 2e-3
TRACE_EMU_CHAIN = 5e-3
TRACE_F32 = 1e-2


def traced_forward(jc, eng, c, ids, markers, qtype, mode=0, head_rows=0):
    """julia_cuda_forward_trace: (logits, encoder stream [L][n][D], head stream [H + 1][nh][D],
    scorer hidden layer [k][S]) as f32 numpy arrays."""
    n = len(ids)
    nh = head_rows if 0 < head_rows < n else n
    ids_t = torch.from_numpy(np.asarray(ids, np.uint32).view(np.int32)).cuda()
    mk_t = torch.from_numpy(np.asarray(markers, np.uint32).view(np.int32)).cuda()
    logits = torch.zeros(len(markers), dtype=torch.float32, device="cuda")
    f16 = dict(dtype=torch.float16, device="cuda")
    tr = torch.zeros(c.n_layers, n, c.d_model, **f16)
    ht = torch.zeros(c.n_head_layers + 1, nh, c.d_model, **f16)
    st = torch.zeros(len(markers), c.scorer_hidden, **f16)
    eng.forward_trace(ids_t, mk_t, qtype, logits, trace=tr, head_trace=ht, scorer_trace=st,
                      layer_fused=mode)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    return f(logits), f(tr), f(ht), f(st)


def check_traced(O, c, raw, ids, markers, qtype, got, emu_bar, head_rows=0, label=""):
    """Every traced stage and the logits against the emulation and the f32 model; returns the
    worst errors seen (printed by the caller)."""
    logits, tr, ht, st = got
    oc = oracle_cfg(O, c)
    le, tre, hte, ste = O.forward_traced(oc, raw, ids, markers, qtype, head_rows=head_rows,
                                         emulate=True)
    lf, trf, htf, stf = O.forward_traced(oc, raw, ids, markers, qtype, head_rows=head_rows)
    worst = {"enc_emu": 0.0, "enc_f32": 0.0, "head_emu": 0.0, "head_f32": 0.0}
    for l in range(c.n_layers):
        e1, e2 = rel_err(tr[l], tre[l]), rel_err(tr[l], trf[l])
        worst["enc_emu"], worst["enc_f32"] = max(worst["enc_emu"], e1), max(worst["enc_f32"], e2)
        assert e1 < emu_bar and e2 < TRACE_F32, f"{label} encoder layer {l}: {e1:.2e} {e2:.2e}"
    for s in range(c.n_head_layers + 1):
        e1, e2 = rel_err(ht[s], hte[s]), rel_err(ht[s], htf[s])
        worst["head_emu"], worst["head_f32"] = max(worst["head_emu"], e1), max(worst["head_f32"], e2)
        stage = "input" if s == 0 else f"layer {s - 1}"
        assert e1 < emu_bar and e2 < TRACE_F32, f"{label} head {stage}: {e1:.2e} {e2:.2e}"
    worst["scorer_emu"], worst["scorer_f32"] = rel_err(st, ste), rel_err(st, stf)
    assert worst["scorer_emu"] < emu_bar and worst["scorer_f32"] < TRACE_F32, f"{label} scorer {worst}"
    worst["logits_emu"], worst["logits_f32"] = rel_logits(logits, le), rel_logits(logits, lf)
    assert worst["logits_emu"] < LOGIT_REL_EMU, f"{label} logits vs emulation {worst}"
    assert worst["logits_f32"] < LOGIT_REL_F32, f"{label} logits vs f32 {worst}"
    assert np.max(np.abs(logits - lf)) < 0.15 and np.mean(np.abs(logits - lf)) <= 0.03
    assert np.argmax(logits) == np.argmax(lf)
    return worst


def raw_tensor(jc, c, raw, index):
    """A view of tensor `index` (julia_cuda_raw_offsets order) of a raw weight array."""
    off = jc.raw_offsets(c)
    end = int(off[index + 1]) if index + 1 < len(off) else raw.size
    return raw[int(off[index]):end]


def head_l2_bias_index(jc, c):
    """raw_offsets index of the last head layer's linear2 bias: the last of the head layers'
    tensors, followed only by the scorer's six (norm w, b, lin1 w, b, lin2 w, b)."""
    return len(jc.raw_offsets(c)) - 7


def oracle_cfg(O, c):
    return O.Config(*[getattr(c, f) for f, _ in c._fields_])


def small_cfg(jc):
    return jc.default_config(d_model=256, inter=256, n_layers=4, vocab=1000, head_ff=512,
                             scorer_hidden=128, max_positions=2048)


def device_forward(jc, eng, ids, markers, qtype, n_layers, d, trace=True, mode=0):
    ids_t = torch.from_numpy(np.asarray(ids, np.uint32).view(np.int32)).cuda()
    mk_t = torch.from_numpy(np.asarray(markers, np.uint32).view(np.int32)).cuda()
    logits = torch.zeros(len(markers), dtype=torch.float32, device="cuda")
    tr = torch.zeros(n_layers, len(ids), d, dtype=torch.float16, device="cuda") if trace else None
    eng.forward_device(ids_t, mk_t, qtype, logits, trace=tr, layer_fused=mode)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    out = logits.cpu().numpy()
    return (out, tr.float().cpu().numpy()) if trace else out


@pytest.fixture(scope="module")
def small_engine(jc, O):
    c = small_cfg(jc)
    raw = O.init_random(oracle_cfg(O, c), 21)
    eng = jc.Engine.load_raw(c, raw, max_length=1024)
    yield c, raw, eng
    eng.close()


@pytest.mark.parametrize("n,qtype", [(1, 0), (65, 1), (200, 2), (600, 0)])
def test_small_model_forward(jc, O, small_engine, n, qtype):
    c, raw, eng = small_engine
    rng = np.random.default_rng(n)
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.unique(rng.integers(0, n, 4)).astype(np.uint32)
    got, tr = device_forward(jc, eng, ids, markers, qtype, c.n_layers, c.d_model)
    oc = oracle_cfg(O, c)
    emu, tr_emu = O.forward_emu(oc, raw, ids, markers, qtype, trace=True)
    f32, tr_f32 = O.forward_f32(oc, raw, ids, markers, qtype, trace=True)
    for l in range(c.n_layers):
        assert rel_err(tr[l], tr_emu[l]) < 5e-3, f"layer {l} vs emulation"
        assert rel_err(tr[l], tr_f32[l]) < 3e-2, f"layer {l} vs f32"
    assert np.max(np.abs(got - emu)) < 2e-3
    assert np.max(np.abs(got - f32)) < 0.15 and np.mean(np.abs(got - f32)) <= 0.03
    # The graph path against the traced (ungraphed) path: the same kernels; only the order of the
    # row statistics' atomic additions differs between runs.
    again = device_forward(jc, eng, ids, markers, qtype, c.n_layers, c.d_model, trace=False)
    assert np.max(np.abs(again - got)) < 1e-3


@pytest.fixture(scope="module")
def full_engine(jc, O):
    c = jc.default_config(max_positions=1024)
    raw = O.init_random(oracle_cfg(O, c), 1234)
    eng = jc.Engine.load_raw(c, raw, max_length=1024)
    yield c, raw, eng
    eng.close()


def test_benchmark_config_293_tokens(jc, O, full_engine):
    """hidden 768, 12 heads, 22 layers, 293 tokens, 4 markers."""
    c, raw, eng = full_engine
    rng = np.random.default_rng(293)
    ids = rng.integers(0, c.vocab, 293).astype(np.uint32)
    markers = np.sort(rng.choice(293, 4, replace=False)).astype(np.uint32)
    got, tr = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model)
    oc = oracle_cfg(O, c)
    f32, tr_f32 = O.forward_f32(oc, raw, ids, markers, 0, trace=True)
    emu = O.forward_emu(oc, raw, ids, markers, 0)
    worst = max(rel_err(tr[l], tr_f32[l]) for l in range(c.n_layers))
    assert worst < 3e-2, worst
    assert np.max(np.abs(got - emu)) < 2e-3
    assert np.max(np.abs(got - f32)) < 0.15 and np.mean(np.abs(got - f32)) <= 0.03
    assert np.argmax(got) == np.argmax(f32)


def test_run_batch_matches_device_path(jc, O, full_engine):
    """julia_cuda_run (host arrays, queued back to back) against one-at-a-time device calls."""
    c, raw, eng = full_engine
    rng = np.random.default_rng(5)
    seqs = []
    for i, n in enumerate([293, 32, 1024, 77, 293, 500]):
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        mk = np.sort(rng.choice(n, min(4, n), replace=False)).astype(np.uint32)
        seqs.append((ids, mk, i % 3))
    outs, ms = eng.run(seqs)
    assert np.all(ms > 0)
    for (ids, mk, q), got in zip(seqs, outs):
        want = device_forward(jc, eng, ids, mk, q, c.n_layers, c.d_model, trace=False)
        assert np.max(np.abs(got - want)) < 1e-3


def test_argmax_agreement_on_serving_lengths(jc, O, full_engine):
    """Log-normal lengths (BASELINE config 3's distribution), argmax vs the f32 model."""
    c, raw, eng = full_engine
    rng = np.random.default_rng(2024)
    sigma = 0.5
    lens = np.clip(np.round(rng.lognormal(np.log(293) - sigma ** 2 / 2, sigma, 12)), 32,
                   1024).astype(int)
    oc = oracle_cfg(O, c)
    seqs = []
    for i, n in enumerate(lens):
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        mk = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
        seqs.append((ids, mk, i % 3))
    outs, _ = eng.run(seqs)
    diffs, agree = [], 0
    for (ids, mk, q), got in zip(seqs, outs):
        want = O.forward_f32(oc, raw, ids, mk, q)
        diffs.append(np.abs(got - want))
        agree += int(np.argmax(got) == np.argmax(want))
    d = np.concatenate(diffs)
    assert d.max() < 0.15 and d.mean() <= 0.03
    assert agree == len(seqs)


def test_run_rejects_bad_requests(jc, full_engine):
    c, raw, eng = full_engine
    ok = (np.arange(10, dtype=np.uint32), np.array([1], np.uint32), 0)
    with pytest.raises(jc.JuliaCudaError, match="tokens"):
        eng.run([ok, (np.zeros(0, np.uint32), np.zeros(0, np.uint32), 0)])
    with pytest.raises(jc.JuliaCudaError, match="tokens"):
        eng.run([(np.zeros(1025, np.uint32), np.array([0], np.uint32), 0)])
    with pytest.raises(jc.JuliaCudaError, match="marker"):
        eng.run([(np.arange(10, dtype=np.uint32), np.array([10], np.uint32), 0)])
    with pytest.raises(jc.JuliaCudaError, match="question type"):
        eng.run([(np.arange(10, dtype=np.uint32), np.array([1], np.uint32), 3)])
    with pytest.raises(jc.JuliaCudaError, match="vocabulary"):
        eng.run([(np.array([c.vocab], np.uint32), np.array([0], np.uint32), 0)])
    # the engine still works after rejected requests
    outs, _ = eng.run([ok])
    assert np.isfinite(outs[0]).all()


def test_reference_width_engine(jc, O):
    """The reference's own Julia-1 width: 384 hidden, 6 heads, scorer 384 -> 384 -> 1."""
    c = jc.default_config(d_model=384, scorer_hidden=384, n_layers=4, vocab=2000,
                          max_positions=512)
    raw = O.init_random(oracle_cfg(O, c), 8)
    eng = jc.Engine.load_raw(c, raw, max_length=512)
    ids = np.arange(363, dtype=np.uint32) * 7 % c.vocab
    mk = np.array([3, 100, 362], np.uint32)
    got, tr = device_forward(jc, eng, ids, mk, 1, c.n_layers, c.d_model)
    f32 = O.forward_f32(oracle_cfg(O, c), raw, ids, mk, 1)
    emu = O.forward_emu(oracle_cfg(O, c), raw, ids, mk, 1)
    assert np.max(np.abs(got - emu)) < 2e-3 and np.max(np.abs(got - f32)) < 0.15
    eng.close()


def test_load_from_directory(jc, O, tmp_path):
    """julia_cuda_load (the reference's entry point) from a saved raw model."""
    import ctypes
    c = small_cfg(jc)
    raw = jc.init_random(c, 77)
    err = ctypes.create_string_buffer(256)
    assert jc.lib().julia_cuda_save_raw(str(tmp_path).encode(), ctypes.byref(c), raw.ctypes.data,
                                        err, 256) == 0
    eng = jc.Engine.load(str(tmp_path), max_length=256)
    assert "B200" in eng.device_name()
    outs, ms = eng.run([(np.arange(50, dtype=np.uint32), np.array([0, 49], np.uint32), 0)])
    want = O.forward_f32(oracle_cfg(O, c), raw, np.arange(50), [0, 49], 0)
    assert np.max(np.abs(outs[0] - want)) < 0.15
    eng.close()


# ---- the persistent kernel: one launch per encoder layer (mode 1), one for the model (mode 2) ----

@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("n,qtype", [(1, 0), (65, 1), (293, 2), (600, 0)])
def test_persistent_modes(jc, O, small_engine, mode, n, qtype):
    """The persistent layer kernel (the reference's layer-fused mode, src/forward.rs:226-359) and
    the whole-model kernel against the emulation and the f32 model, and against the per-step
    kernels (same tiles; only the order of the row statistics' atomic additions differs)."""
    c, raw, eng = small_engine
    rng = np.random.default_rng(n + 7)
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.unique(rng.integers(0, n, 4)).astype(np.uint32)
    got, tr = device_forward(jc, eng, ids, markers, qtype, c.n_layers, c.d_model, mode=mode)
    oc = oracle_cfg(O, c)
    emu, tr_emu = O.forward_emu(oc, raw, ids, markers, qtype, trace=True)
    f32 = O.forward_f32(oc, raw, ids, markers, qtype)
    for l in range(c.n_layers):
        assert rel_err(tr[l], tr_emu[l]) < 5e-3, f"layer {l} vs emulation"
    assert np.max(np.abs(got - emu)) < 2e-3
    assert np.max(np.abs(got - f32)) < 0.15
    steps = device_forward(jc, eng, ids, markers, qtype, c.n_layers, c.d_model, trace=False)
    graphed = device_forward(jc, eng, ids, markers, qtype, c.n_layers, c.d_model, trace=False,
                             mode=mode)
    assert np.max(np.abs(graphed - steps)) < 1e-3


@pytest.mark.parametrize("policy", [32, 64])
@pytest.mark.parametrize("mode", [1, 2])
def test_persistent_tile_widths(jc, O, policy, mode):
    """Every GEMM phase that allows it at one tile width (jc_persist_tile_policy: 32 or 64
    columns; RoPE and GeGLU phases stay 64): the persistent kernel against the emulation and the
    per-step kernels, on a fresh engine (its plans are made under the policy)."""
    c = small_cfg(jc)
    raw = O.init_random(oracle_cfg(O, c), 21)
    old = jc.persist_tile_policy(policy)
    try:
        eng = jc.Engine.load_raw(c, raw, max_length=1024)
        try:
            for n in (65, 293):
                rng = np.random.default_rng(n + policy)
                ids = rng.integers(0, c.vocab, n).astype(np.uint32)
                markers = np.unique(rng.integers(0, n, 4)).astype(np.uint32)
                got, tr = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model, mode=mode)
                emu, tr_emu = O.forward_emu(oracle_cfg(O, c), raw, ids, markers, 0, trace=True)
                for l in range(c.n_layers):
                    assert rel_err(tr[l], tr_emu[l]) < 5e-3, f"layer {l} vs emulation"
                assert np.max(np.abs(got - emu)) < 2e-3
                graphed = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model,
                                         trace=False, mode=mode)
                steps = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model,
                                       trace=False)
                assert np.max(np.abs(graphed - steps)) < 1e-3
        finally:
            eng.close()
    finally:
        assert jc.persist_tile_policy(old) == policy


@pytest.mark.parametrize("mode", [1, 2])
def test_persistent_benchmark_config(jc, O, full_engine, mode):
    c, raw, eng = full_engine
    rng = np.random.default_rng(293)
    ids = rng.integers(0, c.vocab, 293).astype(np.uint32)
    markers = np.sort(rng.choice(293, 4, replace=False)).astype(np.uint32)
    outs, ms = eng.run([(ids, markers, 0)], layer_fused=mode)
    f32 = O.forward_f32(oracle_cfg(O, c), raw, ids, markers, 0)
    assert np.max(np.abs(outs[0] - f32)) < 0.15 and np.argmax(outs[0]) == np.argmax(f32)
    steps, _ = eng.run([(ids, markers, 0)], layer_fused=0)
    assert np.max(np.abs(outs[0] - steps[0])) < 1e-3


def test_grid_barrier_timeout_is_reported(jc, small_engine):
    """Failure detection without a GPU fault: a grid barrier that waits for one CTA more than the
    grid has must give up after its limit (0.2 s here), record JC_DEV_TIMEOUT_GRID (4) and leave
    the engine usable."""
    c, raw, eng = small_engine
    assert eng.barrier_timeout_probe(200_000_000) == 4
    assert jc.device_error() == 0 and eng.device_error() == 0
    ids = np.arange(40, dtype=np.uint32)
    for mode in (0, 1, 2):
        outs, _ = eng.run([(ids, np.array([0, 39], np.uint32), 0)], layer_fused=mode)
        assert np.isfinite(outs[0]).all()


def test_engines_keep_their_own_error_words(jc, O, small_engine):
    """Two engines on one GPU: while one makes a persistent-kernel wait time out on purpose
    (0.3 s), the other serves requests from another host thread. Each reports only its own
    status: the probe's code, none for the serving engine, and nothing in the module's word that
    the bare jc_* entry points use."""
    import threading

    c, raw, eng_a = small_engine
    eng_b = jc.Engine.load_raw(c, raw, max_length=256)
    try:
        ids = np.arange(100, dtype=np.uint32) % c.vocab
        req = [(ids, np.array([0, 50, 99], np.uint32), 1)]
        want, _ = eng_b.run(req)
        probe = {}

        def run_probe():
            probe["code"] = eng_a.barrier_timeout_probe(300_000_000)

        t = threading.Thread(target=run_probe)
        t.start()
        served = []
        while t.is_alive() or len(served) < 3:
            outs, _ = eng_b.run(req, layer_fused=len(served) % 3)
            served.append(outs[0])
        t.join()
        assert probe["code"] == 4
        for got in served:
            assert np.max(np.abs(got - want[0])) < 2e-3
        assert eng_b.device_error() == 0
        assert eng_a.device_error() == 0
        assert jc.device_error() == 0
        outs, _ = eng_a.run(req)
        assert np.max(np.abs(outs[0] - want[0])) < 2e-3
    finally:
        eng_b.close()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_traced_stages_small_model(jc, O, small_engine, mode):
    """Every stage of the small model (4 layers) traced, against the emulation and the f32 model,
    in each execution mode."""
    c, raw, eng = small_engine
    rng = np.random.default_rng(31 + mode)
    n = 293
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
    got = traced_forward(jc, eng, c, ids, markers, mode % 3, mode=mode)
    w = check_traced(O, c, raw, ids, markers, mode % 3, got, TRACE_EMU, label=f"mode {mode}")
    print(f"\nsmall model, mode {mode}: " + ", ".join(f"{k} {v:.2e}" for k, v in w.items()))


def test_traced_stages_benchmark_config(jc, O, full_engine):
    """BASELINE config 0 (hidden 768, 22 layers, 293 tokens) traced stage by stage, and the gate's
    sensitivity: the same comparison against an oracle whose last head layer leaves out its
    linear2 bias (a planted mistake, on the CPU) must fail the bars."""
    c, raw, eng = full_engine
    rng = np.random.default_rng(293)
    ids = rng.integers(0, c.vocab, 293).astype(np.uint32)
    markers = np.sort(rng.choice(293, 4, replace=False)).astype(np.uint32)
    got = traced_forward(jc, eng, c, ids, markers, 0)
    w = check_traced(O, c, raw, ids, markers, 0, got, TRACE_EMU_CHAIN, label="config 0")
    print("\nconfig 0: " + ", ".join(f"{k} {v:.2e}" for k, v in w.items()))
    broken = raw.copy()
    raw_tensor(jc, c, broken, head_l2_bias_index(jc, c))[:] = 0.0
    with pytest.raises(AssertionError):
        check_traced(O, c, broken, ids, markers, 0, got, TRACE_EMU_CHAIN, label="broken bias")


def test_planted_head_bias_mistake_is_visible_in_the_logits(jc, O, full_engine):
    """The logit bars alone (no trace) also catch the planted mistake: the engine's logits against
    the broken oracle's are off by more than LOGIT_REL_EMU."""
    c, raw, eng = full_engine
    rng = np.random.default_rng(294)
    ids = rng.integers(0, c.vocab, 293).astype(np.uint32)
    markers = np.sort(rng.choice(293, 4, replace=False)).astype(np.uint32)
    got = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model, trace=False)
    broken = raw.copy()
    raw_tensor(jc, c, broken, head_l2_bias_index(jc, c))[:] = 0.0
    oc = oracle_cfg(O, c)
    good, bad = O.forward_emu(oc, raw, ids, markers, 0), O.forward_emu(oc, broken, ids, markers, 0)
    print(f"\nlogits vs emulation {rel_logits(got, good):.2e}, vs the broken oracle "
          f"{rel_logits(got, bad):.2e}")
    assert rel_logits(got, good) < LOGIT_REL_EMU
    assert rel_logits(got, bad) > LOGIT_REL_EMU


def test_profiled_forward_stamps_every_phase(jc, O, small_engine):
    """julia_cuda_forward_profile: the same logits as the plain forward, one launch entry per
    kernel of the forward, and in every GEMM CTA's record the phases in order (entry <= inputs
    ready <= first stage <= accumulator <= outputs written <= exit) on a valid SM."""
    c, raw, eng = small_engine
    rng = np.random.default_rng(77)
    n = 293
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
    plain = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model, trace=False)
    ids_t = torch.from_numpy(ids.view(np.int32)).cuda()
    mk_t = torch.from_numpy(markers.view(np.int32)).cuda()
    logits = torch.zeros(4, dtype=torch.float32, device="cuda")
    recs, launches = eng.forward_profile(ids_t, mk_t, 0, logits, records_per_launch=256)
    assert eng.device_error() == 0
    assert np.max(np.abs(logits.cpu().numpy() - plain)) < 1e-3
    assert len(launches) == eng.launches_per_forward(n, 4)
    kinds = [li["kind"] for li in launches]
    assert kinds.count(0) == 4 * c.n_layers + 4 * c.n_head_layers + 1
    assert kinds.count(1) == c.n_layers + c.n_head_layers
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for li in launches:
        if li["kind"] not in (0, 1):
            continue
        assert li["records"] == min(li["ctas"], 256) and li["launch"] == launches.index(li)
        r = recs[li["record"]:li["record"] + li["records"]].astype(np.int64)
        assert (r[:, 0] > 0).all() and (r[:, 6] < sms).all()
        assert np.array_equal(r[:, 7], np.arange(len(r)))
        if li["kind"] == 0:
            assert (np.diff(r[:, :6], axis=1) >= 0).all(), li


@pytest.mark.parametrize("mode", [1, 2])
def test_profiled_persistent_forward_stamps_every_item(jc, O, small_engine, mode):
    """julia_cuda_forward_profile_mode with the persistent kernel: the same logits as the plain
    forward; one entry per phase of every persistent launch (mode 2: one launch, mode 1: one per
    encoder layer beside the per-step edges and head), each owning all of its items' records; in
    every item's record the stages in order (taken <= inputs ready <= reported; a GEMM tile's
    first stage, accumulator and outputs in between) on a valid SM and CTA."""
    c, raw, eng = small_engine
    rng = np.random.default_rng(78)
    n = 293
    ids = rng.integers(0, c.vocab, n).astype(np.uint32)
    markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
    plain = device_forward(jc, eng, ids, markers, 0, c.n_layers, c.d_model, trace=False, mode=mode)
    ids_t = torch.from_numpy(ids.view(np.int32)).cuda()
    mk_t = torch.from_numpy(markers.view(np.int32)).cuda()
    logits = torch.zeros(4, dtype=torch.float32, device="cuda")
    recs, launches = eng.forward_profile(ids_t, mk_t, 0, logits, records_per_launch=256,
                                         layer_fused=mode)
    assert eng.device_error() == 0
    assert np.max(np.abs(logits.cpu().numpy() - plain)) < 1e-3
    assert len({li["launch"] for li in launches}) == eng.launches_per_forward(n, 4, mode)
    phases = [li for li in launches if li["items"]]
    assert len({li["launch"] for li in phases}) == (1 if mode == 2 else c.n_layers)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    gemm_items = 0
    for li in phases:
        assert li["records"] == li["items"], li
        r = recs[li["record"]:li["record"] + li["records"]].astype(np.int64)
        assert (r[:, 0] > 0).all() and (r[:, 1] >= r[:, 0]).all() and (r[:, 5] >= r[:, 1]).all(), li
        assert (r[:, 6] < sms).all() and (r[:, 7] < li["ctas"]).all()
        if li["kind"] == 0:
            gemm_items += len(r)
            assert (np.diff(r[:, :6], axis=1) >= 0).all(), li
    assert gemm_items > 0
