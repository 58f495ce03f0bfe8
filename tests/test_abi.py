"""The C-ABI library on CPU: it loads, exports every symbol include/julia_cuda.h declares, and its
host-side pieces (raw layout, synthetic weights, weight preparation, plan choice, argument
validation) agree with the oracle. No kernel is launched here."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "julia_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b((?:julia_cuda|jc)_[a-z0-9_]+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(jc):
    lib = ctypes.CDLL(jc.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_tier_and_default_config(jc):
    assert jc.lib().julia_cuda_tier() == b"sm_100a"
    c = jc.default_config()
    assert (c.d_model, c.n_heads, c.inter, c.n_layers, c.vocab) == (768, 12, 1152, 22, 50368)
    assert (c.head_ff, c.scorer_hidden, c.n_head_layers, c.global_every, c.window) == (
        2048, 384, 2, 3, 64)
    assert (c.theta_global, c.theta_local) == (160000.0, 10000.0)


def as_oracle(O, c):
    return O.Config(*[getattr(c, f) for f, _ in c._fields_])


@pytest.mark.parametrize("kw", [dict(n_layers=3, vocab=100, head_ff=128, scorer_hidden=64,
                                     d_model=256, inter=192), dict()])
def test_raw_layout_matches_oracle(jc, O, kw):
    c = jc.default_config(**kw)
    oc = as_oracle(O, c)
    assert jc.raw_size(c) == O.raw_size(oc)
    offs = jc.raw_offsets(c)
    assert offs[0] == 0 and np.all(np.diff(offs.astype(np.int64)) >= 0)


def test_init_random_matches_oracle(jc, O):
    c = jc.default_config(n_layers=2, vocab=64, head_ff=128, scorer_hidden=64, d_model=128,
                          inter=128)
    a = jc.init_random(c, 42)
    b = O.init_random(as_oracle(O, c), 42)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # gammas around 1, matrices around 0 with std 0.02
    assert abs(float(a[: 64 * 128].std()) - 0.02) < 2e-3


def test_prep_fold_bit_exact(jc, O):
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (96, 128)).astype(np.float32)
    g = (1 + rng.normal(0, 0.05, 128)).astype(np.float32)
    b = rng.normal(0, 0.02, 128).astype(np.float32)
    bias = rng.normal(0, 0.02, 96).astype(np.float32)
    w16a, csa = jc.prep_fold_layernorm(w, g)
    w16b, csb = O.fold_layernorm(w, g)
    assert np.array_equal(w16a, w16b) and np.array_equal(csa.view(np.uint32), csb.view(np.uint32))
    a = jc.prep_fold_layernorm_bias(w, g, b, bias)
    o = O.fold_layernorm_bias(w, g, b, bias)
    for x, y in zip(a, o):
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8))


def test_prep_rope_table_bit_exact(jc, O):
    for theta in (10000.0, 160000.0):
        a = jc.prep_rope_table(theta, 300)
        b = O.rope_table(theta, 300)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_prep_interleave_geglu_layout(jc):
    """Packed row 64t + 32s + e is GELU input 32t + e (s = 0) or its gate (s = 1)."""
    n, inter = 2304, 1152
    rows = jc.prep_interleave_geglu(np.arange(n, dtype=np.float32))
    for p in range(n):
        t, s, e = p // 64, (p % 64) // 32, p % 32
        assert rows[p] == 32 * t + e + (inter if s else 0)
    w = np.arange(n * 3, dtype=np.uint16).reshape(n, 3)
    assert np.array_equal(jc.prep_interleave_geglu(w)[:, 0], (rows * 3).astype(np.uint16))


def test_prep_rope_gemm_layout(jc, O):
    """jc_gemm's RoPE argument: float4 [16][m], entry (g, r) = (cos, sin) of pairs 2g, 2g + 1."""
    t = O.rope_table(10000.0, 50)
    g = jc.prep_rope_gemm(t, 37)
    assert np.array_equal(g, t[:37].reshape(37, 16, 4).transpose(1, 0, 2))


def test_choose_gemm_fills_the_b200(jc):
    bn, sp = ctypes.c_int(), ctypes.c_int()
    for (m, n, k) in [(293, 2304, 768), (293, 768, 768), (293, 768, 1152), (1024, 2304, 768),
                      (72, 768, 768), (4, 384, 768)]:
        jc.lib().jc_choose_gemm(m, n, k, 148, ctypes.byref(bn), ctypes.byref(sp))
        assert bn.value in (32, 64, 128) and 1 <= sp.value <= 8
        assert n % bn.value == 0 and (k // 64) // sp.value >= 1
        ctas = -(-m // 128) * (n // bn.value) * sp.value
        assert ctas <= 2 * 148
    # The tile widths of the measured sweep up to 1024 tokens; for packs of thousands of rows the
    # widths that measured fastest alone (2304 wide: 128 columns at 3072 rows, 18.9 against 21.4
    # us; 256 at 6144, as CTA pairs, 27.7 against 30.5 us; 768 wide: 128 columns at 6144 rows, 15.0
    # against 18.6 us for one wave of 256).
    want = {(293, 2304): 64, (293, 768): 32, (1024, 2304): 128, (1024, 768): 64, (448, 2304): 64,
            (3072, 2304): 128, (3072, 768): 128, (4096, 2304): 256, (4096, 768): 128,
            (72, 768): 32, (6144, 768): 128, (6144, 2304): 256}
    for (m, n), w in want.items():
        jc.lib().jc_choose_gemm(m, n, 768, 148, ctypes.byref(bn), ctypes.byref(sp))
        assert bn.value == w, (m, n, bn.value)


def test_load_without_gpu_reports_an_error(jc, tmp_path):
    """No crash and a message when the engine cannot be built (no model / no GPU here)."""
    err = ctypes.create_string_buffer(512)
    h = jc.lib().julia_cuda_load(str(tmp_path).encode(), 0, err, 512)
    assert not h and b"no model" in err.value


def test_save_raw_roundtrip_files(jc, tmp_path):
    c = jc.default_config(n_layers=1, vocab=16, head_ff=64, scorer_hidden=64, d_model=128,
                          inter=64)
    raw = jc.init_random(c, 1)
    err = ctypes.create_string_buffer(256)
    rc = jc.lib().julia_cuda_save_raw(str(tmp_path).encode(), ctypes.byref(c),
                                      raw.ctypes.data, err, 256)
    assert rc == 0, err.value
    back = np.fromfile(tmp_path / "jc_weights.f32", np.float32)
    assert np.array_equal(back, raw)


def test_bad_config_rejected(jc):
    c = jc.default_config(d_model=100)
    assert jc.raw_size(c) == 0
    with pytest.raises(jc.JuliaCudaError):
        jc.raw_offsets(c)


def test_layer_rejects_bad_arguments_before_touching_a_gpu(jc):
    """jc_layer (the reference's `layer` kernel boundary): null buffers, a width that is not 64 x
    heads, an inter size that is not a multiple of 64 and a RoPE table shorter than the layer are
    errors with a message, found on the host."""
    lib = jc.lib()
    buf = (ctypes.c_uint16 * 64)()
    f = (ctypes.c_float * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    q = ctypes.cast(f, ctypes.c_void_p)

    def call(x=p, d=768, heads=12, inter=1152, m=293, rope_stride=0, colsum=q):
        return lib.jc_layer(x, p, p, p, q, q, p, colsum, q, rope_stride, p, p, q, p, m, d, heads,
                            inter, 1e-5, 64, None)
    assert call(x=None) == -1 and "null buffer" in jc.last_error()
    assert call(d=760) == -1 and "64 x heads" in jc.last_error()
    assert call(inter=1000) == -1 and "multiple of 64" in jc.last_error()
    assert call(m=0) == -1
    assert call(rope_stride=100) == -1 and "RoPE table" in jc.last_error()
