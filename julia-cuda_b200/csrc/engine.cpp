// The engine: weights on the device, preallocated buffers, and the forward pass as steps.
#include "engine.h"

#include <algorithm>
#include <cstring>

namespace jc {

static constexpr int GRAPH_CACHE = 1024;  // every request length up to 1024 tokens

Engine *Engine::create(const jc_model_config &cfg, const float *raw, size_t max_length,
                       int device, std::string *why) {
    if (!check_config(cfg, why)) return nullptr;
    if (max_length == 0) max_length = (size_t)cfg.max_positions;
    if (max_length > (size_t)cfg.max_positions) {
        *why = "max_length is over the model's max_positions";
        return nullptr;
    }
    Engine *e = new Engine();
    e->cfg = cfg;
    e->device = device;
    e->max_length = max_length;
    if (!e->init(raw, why)) {
        delete e;
        return nullptr;
    }
    return e;
}

Engine::~Engine() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto &kv : graphs) {
        cudaGraphExecDestroy(kv.second.exec);
        if (kv.second.descs) cudaFree(kv.second.descs);
    }
    for (int i = 0; i < QUEUE; i++) {
        if (ev_start[i]) cudaEventDestroy(ev_start[i]);
        if (ev_end[i]) cudaEventDestroy(ev_end[i]);
    }
    for (void *p : allocations) cudaFree(p);
    if (h_ids) cudaFreeHost(h_ids);
    if (h_logits) cudaFreeHost(h_logits);
    if (h_err) cudaFreeHost(h_err);
    if (stream) cudaStreamDestroy(stream);
}

int Engine::add_map(const void *p, uint32_t rows, uint32_t cols, uint32_t box) {
    auto key = std::make_tuple(p, rows, cols, box);
    auto it = map_index.find(key);
    if (it != map_index.end()) return it->second;
    CUtensorMap m;
    if (!make_tmap_f16(&m, p, rows, cols, box)) return -1;
    hmaps.push_back(m);
    map_src.push_back(MapSrc{p, rows, cols});
    map_index.emplace(key, (int)hmaps.size() - 1);
    return (int)hmaps.size() - 1;
}

bool Engine::init(const float *raw, std::string *why) {
    auto cu = [&](cudaError_t err, const char *what) {
        if (err == cudaSuccess) return true;
        *why = std::string(what) + ": " + cudaGetErrorString(err);
        return false;
    };
    int ndev = 0;
    if (!cu(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount")) return false;
    if (device < 0 || device >= ndev) {
        *why = "no GPU " + std::to_string(device);
        return false;
    }
    if (!cu(cudaSetDevice(device), "cudaSetDevice")) return false;
    cudaDeviceProp prop;
    if (!cu(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")) return false;
    if (prop.major != 10 || prop.minor != 0) {
        *why = std::string("the kernels are built for sm_100a (B200); ") + prop.name + " is sm_" +
               std::to_string(prop.major * 10 + prop.minor);
        return false;
    }
    name = prop.name;
    sms = prop.multiProcessorCount;
    if (!cu(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate"))
        return false;

    if (!prepare_weights(cfg, raw, (uint32_t)max_length, &hw, why)) return false;
    auto dalloc = [&](void **p, size_t bytes) {
        if (!cu(cudaMalloc(p, bytes ? bytes : 16), "cudaMalloc")) return false;
        allocations.push_back(*p);
        return true;
    };
    if (!dalloc((void **)&w16, hw.f16.size() * 2) || !dalloc((void **)&w32, hw.f32.size() * 4))
        return false;
    if (!cu(cudaMemcpy(w16, hw.f16.data(), hw.f16.size() * 2, cudaMemcpyHostToDevice), "upload") ||
        !cu(cudaMemcpy(w32, hw.f32.data(), hw.f32.size() * 4, cudaMemcpyHostToDevice), "upload"))
        return false;
    {
        // The GEMM epilogue's RoPE tables (global then local theta), pair-group major with one
        // float4 per (pair group, position), from the arena's [positions][32][2] tables.
        const PreparedLayout &P = hw.layout;
        rope_rows = (uint32_t)max_length;
        std::vector<float> t((size_t)2 * 16 * rope_rows * 4);
        rope_table_gemm(hw.f32.data() + P.rope_global.off, rope_rows, rope_rows, t.data());
        rope_table_gemm(hw.f32.data() + P.rope_local.off, rope_rows, rope_rows,
                        t.data() + (size_t)16 * rope_rows * 4);
        if (!dalloc((void **)&rope_t, t.size() * 4) ||
            !cu(cudaMemcpy(rope_t, t.data(), t.size() * 4, cudaMemcpyHostToDevice), "upload"))
            return false;
    }
    hw.f16.clear();
    hw.f16.shrink_to_fit();
    hw.f32.clear();
    hw.f32.shrink_to_fit();

    const size_t L = max_length, D = cfg.d_model, I = cfg.inter, F = cfg.head_ff,
                 S = cfg.scorer_hidden;
    const size_t rows = (L + 127) / 128 * 128;
    const size_t wide = std::max(I, F);
    bool ok = dalloc((void **)&x, rows * D * 2) && dalloc((void **)&qkv, rows * 3 * D * 2) &&
              dalloc((void **)&o, rows * D * 2) && dalloc((void **)&mb, rows * wide * 2) &&
              dalloc((void **)&hx, rows * D * 2) && dalloc((void **)&xs, rows * D * 2) &&
              dalloc((void **)&ys, rows * S * 2) && dalloc((void **)&stats_a, rows * 8) &&
              dalloc((void **)&stats_b, rows * 8) && dalloc((void **)&stats_s, rows * 8) &&
              dalloc((void **)&ids, input_words() * 4) &&
              dalloc((void **)&iota, L * 4) && dalloc((void **)&logits, L * 4) &&
              dalloc((void **)&dev_err, 16);
    if (!ok || !cu(cudaMemset(dev_err, 0, 16), "memset")) return false;
    markers = ids + L;
    seg = reinterpret_cast<uint2 *>(ids + 2 * L);
    tiles = reinterpret_cast<uint2 *>(ids + 4 * L);
    // Split-K scratch for up to 8 splits of the widest GEMM, split-KV scratch for up to 8 ranges.
    const size_t widest = std::max({3 * D, 2 * I, F, S});
    gemm_ws_cap = rows * widest * 8;
    gemm_cnt_cap = 8192;
    attn_ws_cap = attn_ws_floats((uint32_t)L, cfg.n_heads, 8);
    attn_cnt_cap = attn_counters((uint32_t)L, cfg.n_heads);
    ok = dalloc((void **)&gemm_ws, gemm_ws_cap * 4) && dalloc((void **)&gemm_cnt, gemm_cnt_cap * 4) &&
         dalloc((void **)&attn_ws, attn_ws_cap * 4) && dalloc((void **)&attn_cnt, attn_cnt_cap * 4);
    if (!ok) return false;
    if (!cu(cudaMemset(gemm_cnt, 0, gemm_cnt_cap * 4), "memset") ||
        !cu(cudaMemset(attn_cnt, 0, attn_cnt_cap * 4), "memset") ||
        !cu(cudaMemset(x, 0, rows * D * 2), "memset") ||
        !cu(cudaMemset(o, 0, rows * D * 2), "memset") ||
        !cu(cudaMemset(mb, 0, rows * wide * 2), "memset") ||
        !cu(cudaMemset(hx, 0, rows * D * 2), "memset") || !cu(cudaMemset(xs, 0, rows * D * 2), "memset"))
        return false;
    std::vector<uint32_t> io(L);
    for (size_t i = 0; i < L; i++) io[i] = (uint32_t)i;
    if (!cu(cudaMemcpy(iota, io.data(), L * 4, cudaMemcpyHostToDevice), "upload")) return false;

    // Tensor maps: A operands over the whole (row-padded) activation buffers (128-row boxes),
    // weights in 64-row boxes (the persistent kernel's tile width).
    const PreparedLayout &P = hw.layout;
    m_x = add_map(x, rows, D, 128);
    m_o = add_map(o, rows, D, 128);
    m_m = add_map(mb, rows, I, 128);
    m_f = add_map(mb, rows, F, 128);
    m_hx = add_map(hx, rows, D, 128);
    m_xs = add_map(xs, rows, D, 128);
    for (const LayerSpans &ls : P.layers)
        lmaps.push_back({add_map(w16 + ls.wqkv.off, 3 * D, D, 64), add_map(w16 + ls.wo.off, D, D, 64),
                         add_map(w16 + ls.wi.off, 2 * I, D, 64),
                         add_map(w16 + ls.wo_mlp.off, D, I, 64)});
    for (const HeadSpans &h : P.head)
        hmaps_head.push_back({add_map(w16 + h.in_w.off, 3 * D, D, 64),
                              add_map(w16 + h.out_w.off, D, D, 64), add_map(w16 + h.l1_w.off, F, D, 64),
                              add_map(w16 + h.l2_w.off, D, F, 64)});
    m_s1 = add_map(w16 + P.s_lin1_w.off, S, D, 64);
    if (m_x < 0 || m_o < 0 || m_m < 0 || m_f < 0 || m_hx < 0 || m_xs < 0 || m_s1 < 0) {
        *why = last_error();
        return false;
    }
    // The persistent kernel's narrow (32-column) phases read their weights in 32-row boxes: every
    // weight matrix of an epilogue that may run narrow also gets that map (plan_steps picks the
    // map of the width the plan chose, so a box always matches its stage slot).
    {
        std::vector<std::tuple<const void *, uint32_t, uint32_t>> narrow;
        for (const LayerSpans &ls : P.layers) {
            narrow.emplace_back(w16 + ls.wo.off, D, D);
            narrow.emplace_back(w16 + ls.wo_mlp.off, D, I);
        }
        for (const HeadSpans &h : P.head) {
            narrow.emplace_back(w16 + h.in_w.off, 3 * D, D);
            narrow.emplace_back(w16 + h.out_w.off, D, D);
            narrow.emplace_back(w16 + h.l1_w.off, F, D);
            narrow.emplace_back(w16 + h.l2_w.off, D, F);
        }
        narrow.emplace_back(w16 + P.s_lin1_w.off, S, D);
        for (const auto &t : narrow)
            if (add_map(std::get<0>(t), std::get<1>(t), std::get<2>(t), 32) < 0) {
                *why = last_error();
                return false;
            }
    }
    for (auto &lm : lmaps)
        if (lm.wqkv < 0 || lm.wo < 0 || lm.wi < 0 || lm.wo_mlp < 0) {
            *why = last_error();
            return false;
        }
    if (!dalloc((void **)&dmaps, hmaps.size() * sizeof(CUtensorMap)) ||
        !cu(cudaMemcpy(dmaps, hmaps.data(), hmaps.size() * sizeof(CUtensorMap),
                       cudaMemcpyHostToDevice),
            "upload tensor maps"))
        return false;
    scratch_cap = 16 + 6 * (size_t)cfg.n_layers + 7 * (size_t)cfg.n_head_layers + 10;
    if (!dalloc((void **)&scratch_descs, scratch_cap * sizeof(PhaseDesc))) return false;
    flow_blocks = (uint32_t)(rows / FLOW_BLOCK);
    const size_t words = flow_counter_words((uint32_t)scratch_cap, flow_blocks);
    if (!dalloc((void **)&flow_ctr, words * 4) || !cu(cudaMemset(flow_ctr, 0, words * 4), "memset"))
        return false;
    persist_grid = (uint32_t)(sms * std::max(0, persist_blocks_per_sm()));

    if (!cu(cudaMallocHost((void **)&h_ids, QUEUE * input_words() * 4), "cudaMallocHost") ||
        !cu(cudaMallocHost((void **)&h_logits, QUEUE * L * 4), "cudaMallocHost") ||
        !cu(cudaMallocHost((void **)&h_err, sizeof(unsigned int)), "cudaMallocHost"))
        return false;
    for (int i = 0; i < QUEUE; i++)
        if (!cu(cudaEventCreate(&ev_start[i]), "cudaEventCreate") ||
            !cu(cudaEventCreate(&ev_end[i]), "cudaEventCreate"))
            return false;
    return cu(cudaDeviceSynchronize(), "upload sync");
}

const CUtensorMap *Engine::wmap(const void *p, uint32_t rows, uint32_t cols, int bn) {
    auto key = std::make_tuple(p, rows, cols, bn);
    auto it = wmaps.find(key);
    if (it != wmaps.end()) return &it->second;
    CUtensorMap m;
    if (!make_tmap_f16(&m, p, rows, cols, (uint32_t)bn)) return nullptr;
    return &wmaps.emplace(key, m).first->second;
}

// ---------------------------------------------------------------------------------------------
// the forward pass as steps

Step Engine::gemm_step(uint32_t epi, int map_a, int map_w, const void *w, uint32_t m, uint32_t n,
                       uint32_t k, __half *c, const __half *res, const float *stats_in,
                       const float *colsum, float *stats_out, float *zero, uint32_t zero_len,
                       const float *rope, const float *bias, float eps, int layer) const {
    Step st;
    st.d.kind = PH_GEMM;
    st.d.epi = epi;
    GemmParams &g = st.d.g;
    g.map_a = dmaps + map_a;
    g.map_w = dmaps + map_w;
    g.c = c;
    g.res = res;
    g.ws = gemm_ws;
    g.counters = gemm_cnt;
    g.stats_in = stats_in;
    g.colsum = colsum;
    g.stats_out = stats_out;
    g.zero = zero;
    g.rope = rope;
    g.rope_stride = rope_rows;
    g.bias = bias;
    g.zero_len = zero_len;
    g.m = m;
    g.n = n;
    g.k = k;
    g.eps = eps;
    g.err = dev_err;
    st.map_a = map_a;
    st.w = w;
    st.layer = layer;
    return st;
}

std::vector<Step> Engine::build_steps(uint32_t n, uint32_t k, uint32_t qtype, const Trace &tr,
                                      int mode, bool packed) const {
    std::vector<Step> steps = build_steps_flat(n, k, qtype, tr, mode);
    for (size_t i = 0; i < steps.size(); i++) {
        Step &st = steps[i];
        st.slot = (int)i;
        // Per-step launches stamp per CTA (the persistent kernel stamps per item itself).
        if (tr.prof && (mode == MODE_STEPS || (mode == MODE_LAYER && st.layer < 0))) {
            uint64_t *rec = tr.prof + (size_t)i * tr.prof_cap * 8;
            if (st.d.kind == PH_GEMM) st.d.g.prof = rec, st.d.g.prof_cap = tr.prof_cap;
            if (st.d.kind == PH_ATTN) st.d.a.prof = rec, st.d.a.prof_cap = tr.prof_cap;
        }
    }
    if (packed)
        for (Step &st : steps) {
            // Request-aligned tiles for global attention only: a window already bounds a tile's
            // keys, and splitting its tiles at requests only adds partial ones.
            if (st.d.kind == PH_ATTN) st.d.a.seg = seg, st.d.a.tiles = st.d.a.window ? nullptr : tiles;
            if (st.d.kind == PH_GEMM && (st.d.epi & JC_EPI_ROPE)) st.d.g.seg = seg;
        }
    return steps;
}

std::vector<Step> Engine::build_steps_flat(uint32_t n, uint32_t k, uint32_t qtype,
                                           const Trace &tr, int mode) const {
    uint16_t *d_trace = tr.enc;
    const PreparedLayout &P = hw.layout;
    const uint32_t D = cfg.d_model, I = cfg.inter, F = cfg.head_ff, S = cfg.scorer_hidden;
    std::vector<Step> steps;
    auto row_step = [&](uint32_t kind, int layer) {
        Step st;
        st.d.kind = kind;
        st.layer = layer;
        return st;
    };
    // A copy of `rows` rows of `width` columns into a trace buffer (a row phase in the persistent
    // kernel, a device-to-device copy otherwise).
    auto copy_step = [&](const __half *src, uint16_t *dst, uint32_t rows, uint32_t width, int layer) {
        Step st;
        st.d.kind = PH_COPY;
        st.layer = layer;
        st.d.r.x = src;
        st.d.r.out = reinterpret_cast<__half *>(dst);
        st.d.r.n = rows;
        st.d.r.d = width;
        return st;
    };
    auto attn_step = [&](uint32_t rows, uint32_t window, int layer) {
        Step st;
        st.d.kind = PH_ATTN;
        st.d.a = AttnParams{qkv, o, attn_ws, attn_cnt, rows, (uint32_t)cfg.n_heads, window, nullptr,
                            dev_err};
        st.layer = layer;
        return st;
    };
    {
        Step st = row_step(PH_EMBED, -1);
        RowParams &r = st.d.r;
        r.x = reinterpret_cast<const __half *>(w16 + P.tok_emb.off);
        r.rows = ids;
        r.gamma = w32 + P.emb_norm.off;
        r.out = x;
        r.n = n;
        r.d = D;
        r.eps = cfg.norm_eps;
        steps.push_back(st);
    }
    for (int l = 0; l < cfg.n_layers; l++) {
        const LayerSpans &ls = P.layers[l];
        const LayerMaps &lm = lmaps[l];
        const float *rope = rope_t + (ls.global ? 0 : (size_t)16 * rope_rows * 4);
        // qkv: LayerNorm folded (from layer 1) + RoPE; clears stats_a for wo.
        steps.push_back(gemm_step(ls.has_ln ? (JC_EPI_LN | JC_EPI_ROPE) : JC_EPI_ROPE, m_x, lm.wqkv,
                                  w16 + ls.wqkv.off, n, 3 * D, D, qkv, nullptr, stats_b,
                                  ls.has_ln ? w32 + ls.qkv_colsum.off : nullptr, nullptr, stats_a,
                                  2 * n, rope, nullptr, cfg.norm_eps, l));
        steps.push_back(attn_step(n, ls.global ? 0 : (uint32_t)cfg.window, l));
        // wo: x += o . Wo^T, row statistics into stats_a.
        steps.push_back(gemm_step(JC_EPI_RES | JC_EPI_STATS, m_o, lm.wo, w16 + ls.wo.off, n, D, D,
                                  x, x, nullptr, nullptr, stats_a, nullptr, 0, nullptr, nullptr,
                                  0.f, l));
        // wi: m = GeGLU(LN(x) . Wi^T); clears stats_b for wo_mlp.
        steps.push_back(gemm_step(JC_EPI_LN | JC_EPI_GEGLU, m_x, lm.wi, w16 + ls.wi.off, n, 2 * I, D,
                                  mb, nullptr, stats_a, w32 + ls.wi_colsum.off, nullptr, stats_b,
                                  2 * n, nullptr, nullptr, cfg.norm_eps, l));
        // wo_mlp: x += m . Wo_mlp^T, row statistics into stats_b.
        steps.push_back(gemm_step(JC_EPI_RES | JC_EPI_STATS, m_m, lm.wo_mlp, w16 + ls.wo_mlp.off, n,
                                  D, I, x, x, nullptr, nullptr, stats_b, nullptr, 0, nullptr,
                                  nullptr, 0.f, l));
        if (d_trace && mode == MODE_MODEL) {
            Step st = row_step(PH_COPY, l);
            st.d.r.x = x;
            st.d.r.out = reinterpret_cast<__half *>(d_trace) + (size_t)l * n * D;
            st.d.r.n = n;
            st.d.r.d = D;
            steps.push_back(st);
        }
    }
    // Head input: final LayerNorm + type embedding, statistics into stats_a. The head runs on
    // the first nh rows (all of them unless a head length is set).
    const uint32_t nh = head_rows(n);
    {
        Step st = row_step(PH_NORM_ADD, -2);
        RowParams &r = st.d.r;
        r.x = x;
        r.gamma = w32 + P.final_norm.off;
        r.add = w32 + P.type_emb.off + (size_t)qtype * D;
        r.out = hx;
        r.stats = stats_a;
        r.n = nh;
        r.d = D;
        r.eps = cfg.norm_eps;
        steps.push_back(st);
    }
    if (tr.head) steps.push_back(copy_step(hx, tr.head, nh, D, -2));
    const float heps = cfg.head_eps;
    for (size_t l = 0; l < P.head.size(); l++) {
        const HeadSpans &h = P.head[l];
        const HeadMaps &hm = hmaps_head[l];
        steps.push_back(gemm_step(JC_EPI_LN | JC_EPI_BIAS, m_hx, hm.in, w16 + h.in_w.off, nh, 3 * D, D,
                                  qkv, nullptr, stats_a, w32 + h.in_colsum.off, nullptr, stats_b,
                                  2 * nh, nullptr, w32 + h.in_b.off, heps, -2));
        steps.push_back(attn_step(nh, 0, -2));
        steps.push_back(gemm_step(JC_EPI_BIAS | JC_EPI_RES | JC_EPI_STATS, m_o, hm.out,
                                  w16 + h.out_w.off, nh, D, D, hx, hx, nullptr, nullptr, stats_b,
                                  nullptr, 0, nullptr, w32 + h.out_b.off, 0.f, -2));
        steps.push_back(gemm_step(JC_EPI_LN | JC_EPI_BIAS | JC_EPI_RELU, m_hx, hm.l1, w16 + h.l1_w.off,
                                  nh, F, D, mb, nullptr, stats_b, w32 + h.l1_colsum.off, nullptr,
                                  stats_a, 2 * nh, nullptr, w32 + h.l1_b.off, heps, -2));
        steps.push_back(gemm_step(JC_EPI_BIAS | JC_EPI_RES | JC_EPI_STATS, m_f, hm.l2,
                                  w16 + h.l2_w.off, nh, D, F, hx, hx, nullptr, nullptr, stats_a,
                                  nullptr, 0, nullptr, w32 + h.l2_b.off, 0.f, -2));
        if (tr.head) steps.push_back(copy_step(hx, tr.head + (l + 1) * (size_t)nh * D, nh, D, -2));
    }
    if (k == 0) return steps;
    // Scorer on the marker rows only (rows do not interact after the head's last attention).
    {
        Step st = row_step(PH_GATHER, -2);
        RowParams &r = st.d.r;
        r.x = hx;
        r.rows = markers;
        r.stats_in = stats_a;
        r.out = xs;
        r.stats = stats_s;
        r.n = k;
        r.d = D;
        r.limit = nh;
        steps.push_back(st);
    }
    steps.push_back(gemm_step(JC_EPI_LN | JC_EPI_BIAS | JC_EPI_GELU, m_xs, m_s1,
                              w16 + P.s_lin1_w.off, k, S, D, ys, nullptr, stats_s,
                              w32 + P.s_lin1_colsum.off, nullptr, nullptr, 0, nullptr,
                              w32 + P.s_lin1_b.off, heps, -2));
    if (tr.scorer) steps.push_back(copy_step(ys, tr.scorer, k, S, -2));
    {
        Step st = row_step(PH_SCORE, -2);
        RowParams &r = st.d.r;
        r.x = ys;
        r.rows = iota;
        r.w = reinterpret_cast<const __half *>(w16 + P.s_lin2_w.off);
        r.b = P.s_lin2_b;
        r.logits = logits;
        r.n = k;
        r.d = S;
        steps.push_back(st);
    }
    return steps;
}

bool Engine::run_step(const Step &st, cudaStream_t s) {
    const PhaseDesc &d = st.d;
    jc_launch_info info{};
    info.kind = d.kind;
    info.layer = st.layer;
    const uint32_t cap = d.kind == PH_GEMM ? d.g.prof_cap : d.kind == PH_ATTN ? d.a.prof_cap : 0;
    info.record = (uint32_t)std::max(st.slot, 0) * cap;
    auto logged = [&](bool ok) {
        if (ok && launch_log) {
            info.launch = launch_log->empty() ? 0 : launch_log->back().launch + 1;
            info.records = std::min(info.ctas, cap);
            launch_log->push_back(info);
        }
        return ok;
    };
    switch (d.kind) {
        case PH_GEMM: {
            const GemmParams &p = d.g;
            GemmConfig c = choose_gemm(p.m, p.n, p.k, sms);
            if ((d.epi & (JC_EPI_ROPE | JC_EPI_GEGLU)) && c.bn < 64) {
                c.bn = 64;
                set_gemm_depth(c, p.m, p.n, sms);
            }
            if (gemm_ws_floats(p.m, p.n, c) > gemm_ws_cap || gemm_counters(p.m, p.n, c) > gemm_cnt_cap) {
                set_error("engine: split-K scratch too small");
                return false;
            }
            const CUtensorMap *wm = wmap(st.w, p.n, p.k, (int)gemm_w_rows(c));
            // The A operand in boxes of the tile height (the engine's maps hold 128-row boxes).
            const MapSrc &as = map_src[st.map_a];
            const CUtensorMap *am = c.bm == 128 ? &hmaps[st.map_a] : wmap(as.p, as.rows, as.cols, c.bm);
            if (!wm || !am) return false;
            GemmArgs g;
            g.epi = d.epi;
            g.map_a = *am;
            g.map_w = *wm;
            g.c = p.c;
            g.res = p.res;
            g.ws = p.ws;
            g.counters = p.counters;
            g.stats_in = p.stats_in;
            g.colsum = p.colsum;
            g.stats_out = p.stats_out;
            g.zero = p.zero;
            g.zero_len = p.zero_len;
            g.m = p.m;
            g.n = p.n;
            g.k = p.k;
            g.eps = p.eps;
            g.rope = p.rope;
            g.rope_stride = p.rope_stride;
            g.seg = p.seg;
            g.bias = p.bias;
            g.err = p.err;
            g.prof = p.prof;
            g.prof_cap = p.prof_cap;
            info.epi = d.epi;
            info.m = p.m, info.n = p.n, info.k = p.k;
            info.ctas = gemm_ctas(p.m, p.n, c);
            info.tile = (uint32_t)c.bm << 16 | (uint32_t)c.bn;
            return logged(launch_gemm(g, c, s, true));
        }
        case PH_ATTN: {
            AttnArgs a;
            a.qkv = d.a.qkv;
            a.o = d.a.o;
            a.n = d.a.n;
            a.heads = d.a.heads;
            a.window = d.a.window;
            a.seg = d.a.seg;
            a.tiles = d.a.tiles;
            a.kv_chunks = choose_kv_chunks(a.n, a.heads, a.window, sms, a.seg != nullptr);
            a.ws = attn_ws;
            a.counters = attn_cnt;
            a.err = d.a.err;
            a.prof = d.a.prof;
            a.prof_cap = d.a.prof_cap;
            if (attn_ws_floats(a.n, a.heads, a.kv_chunks) > attn_ws_cap) a.kv_chunks = 1;
            info.m = a.n, info.n = a.heads, info.k = a.window;
            info.ctas = attention_ctas(a);
            return logged(launch_attention(a, s, true));
        }
        // The row-wise edges take no phase stamps: one warp per row, (rows + 3) / 4 CTAs.
        case PH_EMBED:
            info.m = d.r.n, info.n = d.r.d, info.ctas = (d.r.n + 3) / 4;
            return logged(launch_embed(d.r.rows, d.r.n, d.r.x, d.r.gamma, d.r.d, d.r.eps, d.r.out,
                                       d.r.stats, s, true));
        case PH_NORM_ADD:
            info.m = d.r.n, info.n = d.r.d, info.ctas = (d.r.n + 3) / 4;
            return logged(launch_norm_add(d.r.x, d.r.n, d.r.d, d.r.gamma, d.r.add, d.r.eps,
                                          d.r.out, d.r.stats, s, true));
        case PH_GATHER:
            info.m = d.r.n, info.n = d.r.d, info.ctas = (d.r.n + 3) / 4;
            return logged(launch_gather_rows(d.r.x, d.r.stats_in, d.r.d, d.r.rows, d.r.n,
                                             d.r.limit, d.r.out, d.r.stats, s, true, dev_err));
        case PH_SCORE:
            info.m = d.r.n, info.n = d.r.d, info.ctas = (d.r.n + 3) / 4;
            return logged(launch_score(d.r.x, d.r.d, d.r.w, d.r.b, d.r.rows, d.r.n, d.r.logits,
                                       s, true));
        case PH_COPY:
            info.m = d.r.n, info.n = d.r.d;
            return logged(cuda_ok(cudaMemcpyAsync(d.r.out, d.r.x, (size_t)d.r.n * d.r.d * 2,
                                                  cudaMemcpyDeviceToDevice, s),
                                  "copy"));
        default:
            set_error("engine: unknown step");
            return false;
    }
}

void Engine::log_persist(const std::vector<Step> &steps, size_t i, size_t j, uint32_t prof_cap) {
    if (!launch_log) return;
    const uint32_t launch = launch_log->empty() ? 0 : launch_log->back().launch + 1;
    const uint32_t cap = (uint32_t)(j - i) * prof_cap;
    for (size_t t = i; t < j; t++) {
        const PhaseDesc &d = steps[t].d;
        jc_launch_info info{};
        info.kind = d.kind;
        info.epi = d.kind == PH_GEMM ? d.epi : 0;
        if (d.kind == PH_GEMM)
            info.m = d.g.m, info.n = d.g.n, info.k = d.g.k, info.tile = (uint32_t)FLOW_BLOCK << 16 | d.bn;
        else if (d.kind == PH_ATTN)
            info.m = d.a.n, info.n = d.a.heads, info.k = d.a.window;
        else
            info.m = d.r.n, info.n = d.r.d;
        info.layer = steps[t].layer;
        info.ctas = persist_grid;
        info.record = (uint32_t)i * prof_cap + d.first_item;
        info.launch = launch;
        info.records = d.first_item < cap ? std::min(d.items, cap - d.first_item) : 0;
        info.items = d.items;
        launch_log->push_back(info);
    }
}

bool Engine::enqueue_steps(const std::vector<Step> &steps, int mode, const PhaseDesc *descs,
                           uint16_t *d_trace, uint32_t n, cudaStream_t s, uint64_t *prof,
                           uint32_t prof_cap) {
    const uint32_t D = cfg.d_model;
    auto trace_copy = [&](int l) {
        return cuda_ok(cudaMemcpyAsync(d_trace + (size_t)l * n * D, x, (size_t)n * D * 2,
                                       cudaMemcpyDeviceToDevice, s),
                       "trace copy");
    };
    // A persistent launch of steps [i, j): its items' records (profiling runs) start at step i's.
    auto persist = [&](size_t i, size_t j) {
        uint64_t *pr = prof ? prof + (size_t)i * prof_cap * 8 : nullptr;
        if (!launch_persist(descs + i, (uint32_t)(j - i), steps[i].flow_total, flow_ctr, flow_blocks,
                            persist_grid, barrier_timeout_ns, s, dev_err, pr,
                            (uint32_t)(j - i) * prof_cap))
            return false;
        if (prof) log_persist(steps, i, j, prof_cap);
        return true;
    };
    if (mode == MODE_MODEL) return persist(0, steps.size());
    size_t i = 0;
    while (i < steps.size()) {
        const int layer = steps[i].layer;
        if (mode == MODE_LAYER && layer >= 0) {
            size_t j = i;
            while (j < steps.size() && steps[j].layer == layer) j++;
            if (!persist(i, j)) return false;
            i = j;
        } else {
            if (!run_step(steps[i], s)) return false;
            i++;
        }
        if (d_trace && layer >= 0 && (i == steps.size() || steps[i].layer != layer) &&
            !trace_copy(layer))
            return false;
    }
    return true;
}

bool Engine::enqueue_forward(uint32_t n, uint32_t k, uint32_t qtype, int mode,
                             const Trace &tr, cudaStream_t s) {
    if (n == 0 || n > max_length || k > max_length || qtype >= (uint32_t)cfg.n_qtypes) {
        set_error("engine: sequence length, marker count or question type out of range");
        return false;
    }
    if (mode < MODE_STEPS || mode > MODE_MODEL) {
        set_error("engine: no such execution mode");
        return false;
    }
    if (mode != MODE_STEPS && persist_grid == 0) {
        set_error("engine: the persistent kernel cannot be resident on this GPU");
        return false;
    }
    std::vector<Step> steps = build_steps(n, k, qtype, tr, mode);
    if (mode != MODE_STEPS) {
        if (!plan_steps(steps, mode)) return false;
        if (steps.size() > scratch_cap) {
            set_error("engine: too many phases");
            return false;
        }
        std::vector<PhaseDesc> descs(steps.size());
        for (size_t i = 0; i < steps.size(); i++) descs[i] = steps[i].d;
        if (!cuda_ok(cudaMemcpyAsync(scratch_descs, descs.data(), descs.size() * sizeof(PhaseDesc),
                                     cudaMemcpyHostToDevice, s),
                     "phase upload"))
            return false;
        // The copy above is from pageable memory, so it is staged before this call returns.
    }
    return enqueue_steps(steps, mode, scratch_descs, tr.enc, n, s, tr.prof, tr.prof_cap);
}

int Engine::launches_per_forward(uint32_t n, uint32_t k, int mode) const {
    (void)n;
    const int head = 1 + 5 * cfg.n_head_layers + (k ? 3 : 0);
    if (mode == MODE_MODEL) return 1;
    if (mode == MODE_LAYER) return 1 + cfg.n_layers + head;
    return 1 + 5 * cfg.n_layers + head;
}

bool Engine::launch_forward(uint32_t n, uint32_t k, uint32_t qtype, int mode, cudaStream_t s,
                            bool packed) {
    GraphKey key{n, k, qtype, mode, head_rows(n), packed ? 1u : 0u};
    auto it = graphs.find(key);
    if (it == graphs.end()) {
        if (n == 0 || n > max_length || k > max_length || qtype >= (uint32_t)cfg.n_qtypes ||
            mode < MODE_STEPS || mode > MODE_MODEL || (mode != MODE_STEPS && persist_grid == 0)) {
            set_error("engine: sequence length, marker count, question type or mode out of range");
            return false;
        }
        GraphEntry entry;
        std::vector<Step> steps = build_steps(n, k, qtype, Trace{}, mode, packed);
        if (mode != MODE_STEPS) {
            if (!plan_steps(steps, mode)) return false;
            std::vector<PhaseDesc> descs(steps.size());
            for (size_t i = 0; i < steps.size(); i++) descs[i] = steps[i].d;
            if (!cuda_ok(cudaMalloc(&entry.descs, descs.size() * sizeof(PhaseDesc)), "cudaMalloc") ||
                !cuda_ok(cudaMemcpy(entry.descs, descs.data(), descs.size() * sizeof(PhaseDesc),
                                    cudaMemcpyHostToDevice),
                         "phase upload")) {
                if (entry.descs) cudaFree(entry.descs);
                return false;
            }
        }
        cudaStream_t cap = stream;
        if (!cuda_ok(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "begin capture")) {
            if (entry.descs) cudaFree(entry.descs);
            return false;
        }
        const bool ok = enqueue_steps(steps, mode, (const PhaseDesc *)entry.descs, nullptr, n, cap);
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(cap, &graph);
        if (!ok || !cuda_ok(e, "end capture")) {
            if (graph) cudaGraphDestroy(graph);
            if (entry.descs) cudaFree(entry.descs);
            return false;
        }
        e = cudaGraphInstantiate(&entry.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (!cuda_ok(e, "graph instantiate")) {
            if (entry.descs) cudaFree(entry.descs);
            return false;
        }
        // Upload once now, so later launches do not carry the graph's upload.
        if (!cuda_ok(cudaGraphUpload(entry.exec, s), "graph upload")) {
            cudaGraphExecDestroy(entry.exec);
            if (entry.descs) cudaFree(entry.descs);
            return false;
        }
        if ((int)graphs.size() >= GRAPH_CACHE) {
            GraphKey old = graph_lru.back();
            graph_lru.pop_back();
            cudaStreamSynchronize(stream);
            cudaGraphExecDestroy(graphs[old].exec);
            if (graphs[old].descs) cudaFree(graphs[old].descs);
            graphs.erase(old);
        }
        graph_lru.push_front(key);
        entry.lru = graph_lru.begin();
        it = graphs.emplace(key, entry).first;
    } else {
        graph_lru.splice(graph_lru.begin(), graph_lru, it->second.lru);
    }
    return cuda_ok(cudaGraphLaunch(it->second.exec, s), "graph launch");
}

bool Engine::reset_after_error() {
    // A wait that gave up leaves its kernel's counters mid-way: the persistent kernel's
    // dependency counters, and the arrival counters of split-K tiles and split-KV query tiles (a
    // split that timed out never arrives, so a later launch would take the wrong CTA for the
    // last one). Start them all afresh.
    return clear_device_error(dev_err) &&
           cuda_ok(cudaMemsetAsync(flow_ctr, 0, flow_counter_words((uint32_t)scratch_cap, flow_blocks) * 4,
                                   stream),
                   "reset counters") &&
           cuda_ok(cudaMemsetAsync(gemm_cnt, 0, gemm_cnt_cap * 4, stream), "reset counters") &&
           cuda_ok(cudaMemsetAsync(attn_cnt, 0, attn_cnt_cap * 4, stream), "reset counters") &&
           cuda_ok(cudaStreamSynchronize(stream), "reset counters");
}

bool Engine::check_device_error_copy(std::string *why) {
    const unsigned int code = *h_err;
    if (!code) return true;
    if (!reset_after_error()) {
        *why = last_error();
        return false;
    }
    *why = std::string("device error: ") + device_error_name(code);
    return false;
}

bool Engine::take_device_error(unsigned int *code) {
    *code = 0;
    if (!cuda_ok(cudaStreamSynchronize(stream), "sync") || !read_device_error(code, dev_err))
        return false;
    return *code == 0 || reset_after_error();
}

bool Engine::check_device_error(std::string *why) {
    unsigned int code = 0;
    if (!take_device_error(&code)) {
        *why = last_error();
        return false;
    }
    if (code) {
        *why = std::string("device error: ") + device_error_name(code);
        return false;
    }
    return true;
}

bool Engine::barrier_timeout_probe(uint64_t timeout_ns, uint32_t *code) {
    if (persist_grid == 0) {
        set_error("engine: the persistent kernel cannot be resident on this GPU");
        return false;
    }
    // Two row phases (a copy each); the second waits for one item more than the first has, so
    // the wait cannot end and every CTA must give up after timeout_ns.
    std::vector<PhaseDesc> descs(2);
    for (auto &d : descs) {
        d = PhaseDesc{};
        d.kind = PH_COPY;
        d.r.x = x;
        d.r.out = o;
        d.r.n = 1;
        d.r.d = (uint32_t)cfg.d_model;
    }
    const uint32_t total = plan_flow(descs.data(), 2, persist_grid);
    descs[0].extra = 1;
    unsigned int before = 0;
    if (!read_device_error(&before, dev_err)) return false;
    if (!cuda_ok(cudaMemcpy(scratch_descs, descs.data(), 2 * sizeof(PhaseDesc), cudaMemcpyHostToDevice),
                 "phase upload") ||
        !launch_persist(scratch_descs, 2, total, flow_ctr, flow_blocks, persist_grid, timeout_ns, stream,
                        dev_err) ||
        !cuda_ok(cudaStreamSynchronize(stream), "probe"))
        return false;
    unsigned int c = 0;
    if (!read_device_error(&c, dev_err)) return false;
    *code = c;
    return reset_after_error();
}

bool Engine::plan_steps(std::vector<Step> &steps, int mode) const {
    size_t i = 0;
    while (i < steps.size()) {
        size_t j = steps.size();
        if (mode == MODE_LAYER) {
            j = i + 1;
            if (steps[i].layer >= 0)
                while (j < steps.size() && steps[j].layer == steps[i].layer) j++;
        }
        std::vector<PhaseDesc> d(j - i);
        for (size_t t = i; t < j; t++) d[t - i] = steps[t].d;
        const uint32_t total = plan_flow(d.data(), (uint32_t)(j - i), persist_grid);
        for (size_t t = i; t < j; t++) {
            steps[t].d = d[t - i];
            steps[t].flow_total = t == i ? total : 0;
            PhaseDesc &pd = steps[t].d;
            if (pd.kind == PH_GEMM) {
                // The weights' map with boxes as tall as the tile width the plan chose.
                auto it = map_index.find(std::make_tuple(steps[t].w, pd.g.n, pd.g.k, pd.bn));
                if (it == map_index.end()) {
                    set_error("engine: no " + std::to_string(pd.bn) + "-row weight map for a planned phase");
                    return false;
                }
                pd.g.map_w = dmaps + it->second;
            }
        }
        i = j;
    }
    return true;
}

}  // namespace jc
