"""Each sm_100a kernel, called through the C ABI (jc_*), against the oracle's emulation of the
same f16/f32 arithmetic. Tolerances are the reference's (src/check.rs:107, :154, :382-389):
GEMM outputs within 1e-3 relative of the emulation, row statistics 1e-4, attention 2e-3 of the
emulation and 4e-3 of f32, embed within 1 f16 ulp.

A norm-wide bar alone lets a few wrong elements through (one 16-column group of one row off by
30% at 1024 rows moves the Frobenius error by about 1e-3), so every GEMM and attention output is
also bounded element by element, as the reference prints the worst ulp beside the norm
(src/check.rs:147-153): |got - want| <= ELEM x max(|want|, rms(want) / 10) for every element
(ELEM_GEMM 1e-2, about ten f16 ulps; ELEM_ATTN 2e-2)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


ELEM_GEMM = 1e-2
ELEM_ATTN = 2e-2


def elem_err(got, want):
    """Worst element error relative to the element's own size, floored at a tenth of the output's
    rms (elements near zero carry the f32 rounding of their large partial sums)."""
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    floor = 0.1 * max(float(np.sqrt(np.mean(w * w))), 1e-30)
    return float(np.max(np.abs(g - w) / np.maximum(np.abs(w), floor))) if w.size else 0.0


def stats_err(x16, stats):
    """src/check.rs:286-298: max over rows of |dS| / sqrt(S2) and |dS2| / S2."""
    x = x16.view(np.float16).astype(np.float64)
    s_ref = x.sum(1)
    q_ref = np.maximum((x * x).sum(1), 1e-30)
    st = stats.reshape(-1, 2).astype(np.float64)
    return float(np.max(np.maximum(np.abs(st[:, 0] - s_ref) / np.sqrt(q_ref),
                                   np.abs(st[:, 1] - q_ref) / q_ref)))


def ulps(a16, b16):
    def ordered(h):
        h = h.astype(np.int32)
        return np.where(h & 0x8000, -(h & 0x7FFF), h)
    return np.abs(ordered(a16) - ordered(b16))


def cuda_u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)


def cuda_f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host_u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


GEMM_CASES = [
    # name, n, k: BASELINE config 1's encoder GEMMs and the head's variants (hidden 768)
    ("lnrope", 2304, 768),
    ("rope", 2304, 768),
    ("resstats", 768, 768),
    ("lngeglu", 2304, 768),
    ("resstats", 768, 1152),
    ("lnbias", 2304, 768),
    ("lnbiasrelu", 2048, 768),
    ("biasresstats", 768, 2048),
    ("lnbiasgelu", 384, 768),
]


def run_gemm_case(jc, O, name, m, n, k, bn=0, splits=0, seed=0):
    epi = jc.EPILOGUES[name]
    a = O.f16(O.normal((m, k), seed + 1))
    w = O.f16(O.normal((n, k), seed + 2, std=0.05))
    stats_in = O.row_stats(a)
    colsum = O.f32(w).astype(np.float64).sum(1).astype(np.float32)
    rope = O.rope_table(160000.0, max(m, 1))
    bias = O.normal(n, seed + 3, std=0.1)
    res = O.f16(O.normal((m, n), seed + 4))
    want, want_stats = O.emu_gemm(epi, a, w, m, n, k, c16=res if epi & jc.EPI_RES else None,
                                  stats_in=stats_in, colsum=colsum, eps=1e-5, rope=rope,
                                  bias=bias)
    w_dev, cs_dev = w, colsum
    if epi & jc.EPI_GEGLU:
        w_dev = jc.prep_interleave_geglu(w)
        cs_dev = jc.prep_interleave_geglu(colsum)
    n_out = n // 2 if epi & jc.EPI_GEGLU else n
    c = cuda_u16(res) if epi & jc.EPI_RES else torch.zeros(m, n_out, dtype=torch.float16,
                                                         device="cuda")
    stats_out = torch.zeros(2 * m, dtype=torch.float32, device="cuda")
    zero = torch.ones(2 * m + 5, dtype=torch.float32, device="cuda")
    jc.gemm(epi, cuda_u16(a), cuda_u16(w_dev), c, res=c if epi & jc.EPI_RES else None,
            stats_in=cuda_f32(stats_in), colsum=cuda_f32(cs_dev), stats_out=stats_out, zero=zero,
            eps=1e-5, rope=cuda_f32(jc.prep_rope_gemm(rope, m)), bias=cuda_f32(bias), bn=bn,
            splits=splits)
    torch.cuda.synchronize()
    assert jc.device_error() == 0
    got = host_u16(c)
    assert float(zero.abs().max()) == 0.0, "the zero buffer was not cleared"
    e = rel_err(O.f32(got), O.f32(want))
    el = elem_err(O.f32(got), O.f32(want))
    assert e < 1e-3 and el < ELEM_GEMM, (
        f"{name} m={m} n={n} k={k} bn={bn} splits={splits}: rel err {e:.2e}, worst element "
        f"{el:.2e}, worst ulp {int(ulps(got, want).max())}")
    if epi & jc.EPI_STATS:
        se = stats_err(got, stats_out.cpu().numpy())
        assert se < 1e-4, f"{name}: stats err {se:.2e}"
    return e


@pytest.mark.parametrize("name,n,k", GEMM_CASES)
@pytest.mark.parametrize("m", [72, 293, 1024])
def test_gemm_epilogues(jc, O, name, n, k, m):
    run_gemm_case(jc, O, name, m, n, k)


@pytest.mark.parametrize("m", [1, 2, 63, 127, 128, 129, 255, 448])
def test_gemm_ragged_rows(jc, O, m):
    run_gemm_case(jc, O, "lnrope", m, 2304, 768)
    run_gemm_case(jc, O, "resstats", m, 768, 1152)


@pytest.mark.parametrize("name,n,k", [c for c in GEMM_CASES if c[1] % 256 == 0])
@pytest.mark.parametrize("m", [1, 293, 3000])
def test_gemm_256_column_tiles(jc, O, name, n, k, m):
    """256-column tiles (two 256-wide accumulators filling TMEM; what large packs of requests
    take) on every epilogue whose width allows them."""
    run_gemm_case(jc, O, name, m, n, k, bn=256)


PERSISTENT_CASES = [  # (m, tile width): more tiles than SMs, so one CTA per SM walks several
    (1200, 128), (4000, 128), (3000, 256), (6400, 128)]


@pytest.mark.parametrize("name,n,k", GEMM_CASES)
@pytest.mark.parametrize("m,bn", PERSISTENT_CASES)
def test_gemm_persistent_multi_tile(jc, O, name, n, k, m, bn):
    """Launches of more tiles than SMs run the persistent kernel (two TMEM accumulator buffers,
    the epilogue of one tile under the main loop of the next) on every epilogue."""
    tiles = -(-m // 128) * (n // bn) if n % bn == 0 else 0
    if tiles <= 148 or (m >= 4000 and n > 768 and bn == 128):
        pytest.skip("single wave (not the persistent kernel), or a case another row covers")
    run_gemm_case(jc, O, name, m, n, k, bn=bn)


@pytest.fixture
def pairs(jc):
    """Every unsplit 128- or 256-column launch on CTA pairs (jc_gemm_pair_policy 1)."""
    old = jc.gemm_pair_policy(1)
    yield
    assert jc.gemm_pair_policy(old) == 1


PAIR_CASES = [(1, 256), (300, 256), (300, 128), (1000, 128), (3000, 256), (6400, 128)]


@pytest.mark.parametrize("name,n,k", GEMM_CASES)
@pytest.mark.parametrize("m,bn", PAIR_CASES)
def test_gemm_cta_pairs(jc, O, pairs, name, n, k, m, bn):
    """The CTA-pair kernel (tcgen05 cta_group::2: 256-row tiles, each SM of a pair holding 128
    rows and half of the weight tile, the leader issuing every MMA) on every epilogue, at one
    tile, ragged rows (a pair whose second CTA holds no row), one wave and several tiles a pair."""
    if n % bn:
        pytest.skip("the width does not divide n")
    run_gemm_case(jc, O, name, m, n, k, bn=bn)


def test_gemm_pair_policy_hook(jc):
    """jc_gemm_pair_policy returns the previous policy and refuses other values."""
    old = jc.gemm_pair_policy(1)
    try:
        assert jc.gemm_pair_policy(0) == 1
        assert jc.gemm_pair_policy(5) == -2
        assert jc.gemm_pair_policy(-1) == 0
    finally:
        jc.gemm_pair_policy(old)


@pytest.fixture(params=[128, 64])
def tile_rows(request, jc):
    """Both GEMM tile heights: 128 rows, and 64 rows (an M = 64 MMA, its rows in the first 16
    TMEM lanes of each warp quadrant) wherever legal."""
    old = jc.gemm_tile_rows(request.param)
    yield request.param
    jc.gemm_tile_rows(old)


@pytest.mark.parametrize("m", [1, 15, 16, 63, 64, 65, 200, 293, 448, 1024])
def test_gemm_tile_heights(jc, O, tile_rows, m):
    """Every epilogue at ragged row counts with 128- and 64-row tiles (32- and 64-column tiles;
    64-row grids past one wave included)."""
    for name, n, k in GEMM_CASES:
        for bn in ((64,) if name in ("lnrope", "rope", "lngeglu") else (32, 64)):
            run_gemm_case(jc, O, name, m, n, k, bn=bn)


@pytest.mark.parametrize("bn", [32, 64, 128, 256])
@pytest.mark.parametrize("splits", [1, 2, 3, 4, 8])
def test_gemm_tile_and_split_sweep(jc, O, bn, splits):
    """Every tile width x split-K on the resstats and lnbias shapes (the reference's
    configuration sweep, src/check.rs:765-796)."""
    run_gemm_case(jc, O, "resstats", 293, 768, 768, bn=bn, splits=splits)
    run_gemm_case(jc, O, "lnbias", 200, 768, 768, bn=bn, splits=splits)
    if bn >= 64:
        run_gemm_case(jc, O, "lngeglu", 293, 2304, 768, bn=bn, splits=splits)
        run_gemm_case(jc, O, "lnrope", 100, 2304, 768, bn=bn, splits=splits)


def test_gemm_split_k_deterministic(jc, O):
    """Split partials are summed in split order: repeated runs are bit-identical."""
    m, n, k = 293, 768, 1152
    a = cuda_u16(O.f16(O.normal((m, k), 1)))
    w = cuda_u16(O.f16(O.normal((n, k), 2, std=0.05)))
    outs = []
    for _ in range(3):
        c = torch.zeros(m, n, dtype=torch.float16, device="cuda")
        jc.gemm(0, a, w, c, bn=64, splits=4)
        outs.append(host_u16(c))
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("bn", [64, 128])
@pytest.mark.parametrize("cluster", [2, 4])
@pytest.mark.parametrize("m", [1, 129, 293])
def test_gemm_cluster_split(jc, O, bn, cluster, m):
    """Split-K inside a thread-block cluster (splits = -cluster: partials reduced through
    distributed shared memory, no workspace), every epilogue."""
    for name, n, k in GEMM_CASES:
        run_gemm_case(jc, O, name, m, n, k, bn=bn, splits=-cluster)


@pytest.mark.parametrize("bn", [64, 128])
@pytest.mark.parametrize("cluster", [2, 4])
def test_gemm_cluster_split_matches_workspace_split(jc, O, bn, cluster):
    """Both split-K forms sum the same partials in split order from zero, so their outputs are
    bit-identical, and repeated cluster runs are too."""
    m, n, k = 293, 768, 1152
    a = cuda_u16(O.f16(O.normal((m, k), 1)))
    w = cuda_u16(O.f16(O.normal((n, k), 2, std=0.05)))
    res = cuda_u16(O.f16(O.normal((m, n), 3)))
    outs = []
    for splits in (cluster, -cluster, -cluster):
        c = res.clone()
        st = torch.zeros(2 * m, dtype=torch.float32, device="cuda")
        jc.gemm(jc.EPILOGUES["resstats"], a, w, c, res=c, stats_out=st, bn=bn, splits=splits)
        outs.append(host_u16(c))
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


def test_gemm_rejects_bad_cluster(jc):
    a = torch.zeros(10, 128, dtype=torch.float16, device="cuda")
    w = torch.zeros(64, 128, dtype=torch.float16, device="cuda")
    c = torch.zeros(10, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(jc.JuliaCudaError, match="cluster must be 1, 2 or 4"):
        jc.gemm(0, a, w, c, bn=64, splits=-3)
    with pytest.raises(jc.JuliaCudaError, match="cluster split-K needs"):
        jc.gemm(0, a, w, c, bn=32, splits=-2)
    with pytest.raises(jc.JuliaCudaError, match="cluster split-K needs"):
        jc.gemm(0, a, w, c, bn=64, splits=-4)  # k/64 = 2 < 4


def test_gemm_rejects_bad_shapes(jc):
    a = torch.zeros(10, 100, dtype=torch.float16, device="cuda")
    w = torch.zeros(64, 100, dtype=torch.float16, device="cuda")
    c = torch.zeros(10, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(jc.JuliaCudaError, match="multiple of 64"):
        jc.gemm(0, a, w, c)
    a = torch.zeros(10, 128, dtype=torch.float16, device="cuda")
    w = torch.zeros(64, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(jc.JuliaCudaError, match="LayerNorm"):
        jc.gemm(jc.EPI_LN, a, w, c)


@pytest.mark.parametrize("n", [1, 2, 63, 64, 65, 127, 129, 293, 512, 1024])
@pytest.mark.parametrize("window", [0, 64])
def test_attention(jc, O, n, window):
    heads = 12
    qkv = O.f16(O.normal((n, 3 * heads * 64), n + window))
    want = O.emu_attention(qkv, n, heads, window)
    f32 = O.attention_f32(O.f32(qkv), n, heads, window)
    for chunks in ([1, 0, 3] if window == 0 else [1]):
        o = torch.zeros(n, heads * 64, dtype=torch.float16, device="cuda")
        jc.attention(cuda_u16(qkv), o, heads, window, kv_chunks=chunks)
        torch.cuda.synchronize()
        got = O.f32(host_u16(o))
        e1, e2 = rel_err(got, O.f32(want)), rel_err(got, f32)
        el = elem_err(got, O.f32(want))
        assert e1 < 2e-3 and e2 < 4e-3 and el < ELEM_ATTN, \
            f"n={n} window={window} chunks={chunks}: {e1:.2e} {e2:.2e} worst element {el:.2e}"


@pytest.fixture(params=["mma", "tc"])
def attn_kernel(request, jc):
    """Both attention kernels at every length: the mma.sync one (threshold above every length)
    and the tcgen05 one (threshold 1)."""
    t = 0xFFFFFFFF if request.param == "mma" else 1
    old = jc.attention_tc_min(t, t)
    yield request.param
    jc.attention_tc_min(*old)


@pytest.mark.parametrize("n", [1, 2, 63, 65, 129, 200, 293, 1024])
@pytest.mark.parametrize("window", [0, 64])
def test_attention_both_kernels(jc, O, attn_kernel, n, window):
    heads = 12
    qkv = O.f16(O.normal((n, 3 * heads * 64), 3 * n + window))
    want = O.emu_attention(qkv, n, heads, window)
    f32 = O.attention_f32(O.f32(qkv), n, heads, window)
    for chunks in ([1, 0, 3] if window == 0 else [1, 2]):
        o = torch.full((n, heads * 64), float("nan"), dtype=torch.float16, device="cuda")
        jc.attention(cuda_u16(qkv), o, heads, window, kv_chunks=chunks)
        torch.cuda.synchronize()
        assert jc.device_error() == 0
        got = O.f32(host_u16(o))
        e1, e2 = rel_err(got, O.f32(want)), rel_err(got, f32)
        el = elem_err(got, O.f32(want))
        assert e1 < 2e-3 and e2 < 4e-3 and el < ELEM_ATTN, \
            f"{attn_kernel} n={n} window={window} chunks={chunks}: {e1:.2e} {e2:.2e} worst {el:.2e}"


@pytest.mark.parametrize("n,window", [(300, 8), (300, 100), (1024, 200), (700, 31)])
def test_attention_other_windows(jc, O, n, window):
    """Windows narrower and wider than a 64-key tile: the tiles wholly inside every query's
    window skip the mask, the others keep it."""
    heads = 12
    qkv = O.f16(O.normal((n, 3 * heads * 64), 7 * n + window))
    want = O.emu_attention(qkv, n, heads, window)
    o = torch.zeros(n, heads * 64, dtype=torch.float16, device="cuda")
    jc.attention(cuda_u16(qkv), o, heads, window)
    torch.cuda.synchronize()
    got = O.f32(host_u16(o))
    assert rel_err(got, O.f32(want)) < 2e-3 and elem_err(got, O.f32(want)) < ELEM_ATTN


def test_attention_reference_width(jc, O):
    """Six heads (the reference's 384-wide model)."""
    n, heads = 363, 6
    qkv = O.f16(O.normal((n, 3 * heads * 64), 99))
    for window in (0, 64):
        o = torch.zeros(n, heads * 64, dtype=torch.float16, device="cuda")
        jc.attention(cuda_u16(qkv), o, heads, window)
        torch.cuda.synchronize()
        assert rel_err(O.f32(host_u16(o)), O.f32(O.emu_attention(qkv, n, heads, window))) < 2e-3


@pytest.mark.parametrize("d", [384, 768])
def test_embed(jc, O, d):
    vocab, n = 1000, 293
    table = O.f16(O.normal((vocab, d), 5, std=0.02))
    gamma = O.normal(d, 6, mean=1.0, std=0.05)
    ids = np.random.default_rng(0).integers(0, vocab, n).astype(np.uint32)
    want = O.emu_embed(table, gamma, ids, d, 1e-5)
    x = torch.zeros(n, d, dtype=torch.float16, device="cuda")
    stats = torch.zeros(2 * n, dtype=torch.float32, device="cuda")
    jc.embed(torch.from_numpy(ids.view(np.int32)).cuda(), cuda_u16(table), cuda_f32(gamma), x,
             stats=stats)
    torch.cuda.synchronize()
    got = host_u16(x)
    assert ulps(got, want).max() <= 1
    assert stats_err(got, stats.cpu().numpy()) < 1e-4


@pytest.mark.parametrize("d", [384, 768])
def test_norm_add(jc, O, d):
    n = 293
    x = O.f16(O.normal((n, d), 7))
    gamma = O.normal(d, 8, mean=1.0, std=0.05)
    add = O.normal(d, 9, std=0.02)
    want, want_st = O.emu_norm_add(x, gamma, add, 1e-5)
    out = torch.zeros(n, d, dtype=torch.float16, device="cuda")
    st = torch.zeros(2 * n, dtype=torch.float32, device="cuda")
    jc.norm_add(cuda_u16(x), cuda_f32(gamma), cuda_f32(add), out, st)
    torch.cuda.synchronize()
    got = host_u16(out)
    assert ulps(got, want).max() <= 1
    assert stats_err(got, st.cpu().numpy()) < 1e-4


def test_score(jc, O):
    n, d = 293, 384
    y = O.f16(O.normal((n, d), 10))
    w = O.f16(O.normal(d, 11, std=0.05))
    markers = np.array([0, 17, 200, 292, 17], np.uint32)
    want = O.emu_score(y, w, 0.25, markers)
    logits = torch.zeros(len(markers), dtype=torch.float32, device="cuda")
    jc.score(cuda_u16(y), cuda_u16(w), 0.25, torch.from_numpy(markers.view(np.int32)).cuda(),
             logits)
    torch.cuda.synchronize()
    assert np.max(np.abs(logits.cpu().numpy() - want)) < 1e-4


@pytest.mark.parametrize("m,window,ln", [(1, 0, False), (100, 64, True), (293, 0, True),
                                         (293, 64, True), (700, 64, False), (1024, 0, True)])
def test_layer_kernel(jc, O, m, window, ln):
    """jc_layer (the reference's persistent `layer` kernel boundary) against the oracle's emulation
    of the same five steps chained: qkv (LN folded + RoPE, or RoPE alone), attention, wo with
    residual and statistics, wi (LN + GeGLU), wo_mlp with residual and statistics. Every
    intermediate buffer and both statistics buffers are checked."""
    D, H, I, eps = 768, 12, 1152, 1e-5
    x = O.f16(O.normal((m, D), m + 1))
    stats = O.row_stats(x)
    wqkv = O.f16(O.normal((3 * D, D), m + 2, std=0.05))
    qkv_cs = O.f32(wqkv).astype(np.float64).sum(1).astype(np.float32)
    wo = O.f16(O.normal((D, D), m + 3, std=0.05))
    wi = O.f16(O.normal((2 * I, D), m + 4, std=0.05))
    wi_cs = O.f32(wi).astype(np.float64).sum(1).astype(np.float32)
    wo_mlp = O.f16(O.normal((D, I), m + 5, std=0.05))
    rope = O.rope_table(160000.0 if window == 0 else 10000.0, m)
    e_qkv = (jc.EPI_LN | jc.EPI_ROPE) if ln else jc.EPI_ROPE
    qkv_w, _ = O.emu_gemm(e_qkv, x, wqkv, m, 3 * D, D, stats_in=stats, colsum=qkv_cs, eps=eps,
                          rope=rope)
    o_w = O.emu_attention(qkv_w, m, H, window)
    x1, st_a = O.emu_gemm(jc.EPI_RES | jc.EPI_STATS, o_w, wo, m, D, D, c16=x)
    m_w, _ = O.emu_gemm(jc.EPI_LN | jc.EPI_GEGLU, x1, wi, m, 2 * I, D, stats_in=st_a, colsum=wi_cs,
                        eps=eps)
    x2, st_b = O.emu_gemm(jc.EPI_RES | jc.EPI_STATS, m_w, wo_mlp, m, D, I, c16=x1)

    xd = cuda_u16(x)
    qkv_d = torch.zeros(m, 3 * D, dtype=torch.float16, device="cuda")
    o_d = torch.zeros(m, D, dtype=torch.float16, device="cuda")
    m_d = torch.zeros(m, I, dtype=torch.float16, device="cuda")
    st_attn = torch.full((2 * m,), 7.0, dtype=torch.float32, device="cuda")
    st_mlp = cuda_f32(stats.reshape(-1))
    jc.layer(xd, qkv_d, o_d, m_d, st_attn, st_mlp, cuda_u16(wqkv), cuda_f32(qkv_cs) if ln else None,
             cuda_f32(jc.prep_rope_gemm(rope, m)), cuda_u16(wo), cuda_u16(jc.prep_interleave_geglu(wi)),
             cuda_f32(jc.prep_interleave_geglu(wi_cs)), cuda_u16(wo_mlp), H, eps=eps, window=window)
    torch.cuda.synchronize()
    assert jc.device_error() == 0
    for name, got, want, bar in (("qkv", qkv_d, qkv_w, 1e-3), ("o", o_d, o_w, 2e-3),
                                 ("mbuf", m_d, m_w, 3e-3), ("x", xd, x2, 3e-3)):
        g, w = O.f32(host_u16(got)), O.f32(want)
        e, el = rel_err(g, w), elem_err(g, w)
        assert e < bar and el < 5 * ELEM_GEMM, f"{name} m={m} window={window}: {e:.2e} {el:.2e}"
    assert stats_err(host_u16(xd), st_mlp.cpu().numpy()) < 1e-4
    # x1's statistics as the layer computed them, against those of the emulation's x1 (the same
    # values rounded along another path): a row sum's rounding noise scales with the row's norm,
    # so its error is taken relative to sqrt(sum of squares), the sum of squares relative to itself.
    a_rows = st_attn.cpu().numpy().reshape(-1, 2).astype(np.float64)
    x1_rows = np.asarray(st_a, np.float64).reshape(-1, 2)
    sq = np.maximum(x1_rows[:, 1], 1e-30)
    assert np.max(np.abs(a_rows[:, 0] - x1_rows[:, 0]) / np.sqrt(sq)) < 1e-2
    assert np.max(np.abs(a_rows[:, 1] - x1_rows[:, 1]) / sq) < 1e-2
