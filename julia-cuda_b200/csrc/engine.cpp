// The engine: weights on the device, preallocated buffers, and the forward pass.
#include "engine.h"

#include <algorithm>
#include <cstring>

namespace jc {

static constexpr int GRAPH_CACHE = 64;

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
    for (auto &kv : graphs) cudaGraphExecDestroy(kv.second);
    for (int i = 0; i < QUEUE; i++) {
        if (ev_start[i]) cudaEventDestroy(ev_start[i]);
        if (ev_end[i]) cudaEventDestroy(ev_end[i]);
    }
    for (void *p : allocations) cudaFree(p);
    if (h_ids) cudaFreeHost(h_ids);
    if (h_markers) cudaFreeHost(h_markers);
    if (h_logits) cudaFreeHost(h_logits);
    if (stream) cudaStreamDestroy(stream);
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
              dalloc((void **)&ids, L * 4) && dalloc((void **)&markers, L * 4) &&
              dalloc((void **)&iota, L * 4) && dalloc((void **)&logits, L * 4);
    if (!ok) return false;
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
        !cu(cudaMemset(x, 0, rows * D * 2), "memset") || !cu(cudaMemset(o, 0, rows * D * 2), "memset") ||
        !cu(cudaMemset(mb, 0, rows * wide * 2), "memset") ||
        !cu(cudaMemset(hx, 0, rows * D * 2), "memset") || !cu(cudaMemset(xs, 0, rows * D * 2), "memset"))
        return false;
    std::vector<uint32_t> io(L);
    for (size_t i = 0; i < L; i++) io[i] = (uint32_t)i;
    if (!cu(cudaMemcpy(iota, io.data(), L * 4, cudaMemcpyHostToDevice), "upload")) return false;

    // A-operand tensor maps over the whole (row-padded) activation buffers.
    if (!make_tmap_f16(&tm_x, x, rows, D, 128) || !make_tmap_f16(&tm_o, o, rows, D, 128) ||
        !make_tmap_f16(&tm_m, mb, rows, I, 128) || !make_tmap_f16(&tm_f, mb, rows, F, 128) ||
        !make_tmap_f16(&tm_hx, hx, rows, D, 128) || !make_tmap_f16(&tm_xs, xs, rows, D, 128)) {
        *why = last_error();
        return false;
    }

    if (!cu(cudaMallocHost((void **)&h_ids, QUEUE * L * 4), "cudaMallocHost") ||
        !cu(cudaMallocHost((void **)&h_markers, QUEUE * L * 4), "cudaMallocHost") ||
        !cu(cudaMallocHost((void **)&h_logits, QUEUE * L * 4), "cudaMallocHost"))
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

bool Engine::gemm(uint32_t epi, const CUtensorMap &amap, const void *w, uint32_t m, uint32_t n,
                  uint32_t k, __half *c, const __half *res, const float *stats_in,
                  const float *colsum, float *stats_out, float *zero, uint32_t zero_len,
                  const float *rope, const float *bias, float eps, cudaStream_t s) {
    GemmConfig cfgg = choose_gemm(m, n, k, sms);
    if ((epi & (JC_EPI_ROPE | JC_EPI_GEGLU)) && cfgg.bn < 64) {
        cfgg.bn = 64;
        set_gemm_depth(cfgg, m, n, sms);
    }
    GemmArgs g;
    g.epi = epi;
    g.map_a = amap;
    const CUtensorMap *wm = wmap(w, n, k, cfgg.bn);
    if (!wm) return false;
    g.map_w = *wm;
    g.c = c;
    g.res = res;
    g.ws = gemm_ws;
    g.counters = gemm_cnt;
    g.stats_in = stats_in;
    g.colsum = colsum;
    g.stats_out = stats_out;
    g.zero = zero;
    g.zero_len = zero_len;
    g.m = m;
    g.n = n;
    g.k = k;
    g.eps = eps;
    g.rope = rope;
    g.bias = bias;
    if (gemm_ws_floats(m, n, cfgg) > gemm_ws_cap || gemm_counters(m, n, cfgg) > gemm_cnt_cap) {
        set_error("engine: split-K scratch too small");
        return false;
    }
    return launch_gemm(g, cfgg, s, true);
}

bool Engine::attention(const __half *q, __half *out, uint32_t n, uint32_t window, cudaStream_t s) {
    AttnArgs a;
    a.qkv = q;
    a.o = out;
    a.n = n;
    a.heads = cfg.n_heads;
    a.window = window;
    a.kv_chunks = choose_kv_chunks(n, cfg.n_heads, window, sms);
    a.ws = attn_ws;
    a.counters = attn_cnt;
    if (attn_ws_floats(n, cfg.n_heads, a.kv_chunks) > attn_ws_cap) a.kv_chunks = 1;
    return launch_attention(a, s, true);
}

bool Engine::encoder_layer(int l, uint32_t n, cudaStream_t s) {
    const LayerSpans &ls = hw.layout.layers[l];
    const uint32_t D = cfg.d_model, I = cfg.inter;
    const float *rope = w32 + (ls.global ? hw.layout.rope_global.off : hw.layout.rope_local.off);
    // qkv: LayerNorm folded (from layer 1) + RoPE; clears stats_a for wo.
    if (!gemm(ls.has_ln ? (JC_EPI_LN | JC_EPI_ROPE) : JC_EPI_ROPE, tm_x, w16 + ls.wqkv.off, n,
              3 * D, D, qkv, nullptr, stats_b, ls.has_ln ? w32 + ls.qkv_colsum.off : nullptr,
              nullptr, stats_a, 2 * n, rope, nullptr, cfg.norm_eps, s))
        return false;
    if (!attention(qkv, o, n, ls.global ? 0 : (uint32_t)cfg.window, s)) return false;
    // wo: x += o . Wo^T, row statistics into stats_a.
    if (!gemm(JC_EPI_RES | JC_EPI_STATS, tm_o, w16 + ls.wo.off, n, D, D, x, x, nullptr, nullptr,
              stats_a, nullptr, 0, nullptr, nullptr, 0.f, s))
        return false;
    // wi: m = GeGLU(LN(x) . Wi^T); clears stats_b for wo_mlp.
    if (!gemm(JC_EPI_LN | JC_EPI_GEGLU, tm_x, w16 + ls.wi.off, n, 2 * I, D, mb, nullptr, stats_a,
              w32 + ls.wi_colsum.off, nullptr, stats_b, 2 * n, nullptr, nullptr, cfg.norm_eps, s))
        return false;
    // wo_mlp: x += m . Wo_mlp^T, row statistics into stats_b.
    return gemm(JC_EPI_RES | JC_EPI_STATS, tm_m, w16 + ls.wo_mlp.off, n, D, I, x, x, nullptr,
                nullptr, stats_b, nullptr, 0, nullptr, nullptr, 0.f, s);
}

bool Engine::head_and_scorer(uint32_t n, uint32_t k, uint32_t qtype, cudaStream_t s) {
    const PreparedLayout &P = hw.layout;
    const uint32_t D = cfg.d_model, F = cfg.head_ff, S = cfg.scorer_hidden;
    const float eps = cfg.head_eps;
    // Head input: final LayerNorm + type embedding, statistics into stats_a.
    if (!launch_norm_add(x, n, D, w32 + P.final_norm.off, w32 + P.type_emb.off + (size_t)qtype * D,
                         cfg.norm_eps, hx, stats_a, s, true))
        return false;
    for (size_t l = 0; l < P.head.size(); l++) {
        const HeadSpans &h = P.head[l];
        if (!gemm(JC_EPI_LN | JC_EPI_BIAS, tm_hx, w16 + h.in_w.off, n, 3 * D, D, qkv, nullptr,
                  stats_a, w32 + h.in_colsum.off, nullptr, stats_b, 2 * n, nullptr,
                  w32 + h.in_b.off, eps, s))
            return false;
        if (!attention(qkv, o, n, 0, s)) return false;
        if (!gemm(JC_EPI_BIAS | JC_EPI_RES | JC_EPI_STATS, tm_o, w16 + h.out_w.off, n, D, D, hx, hx,
                  nullptr, nullptr, stats_b, nullptr, 0, nullptr, w32 + h.out_b.off, 0.f, s))
            return false;
        if (!gemm(JC_EPI_LN | JC_EPI_BIAS | JC_EPI_RELU, tm_hx, w16 + h.l1_w.off, n, F, D, mb,
                  nullptr, stats_b, w32 + h.l1_colsum.off, nullptr, stats_a, 2 * n, nullptr,
                  w32 + h.l1_b.off, eps, s))
            return false;
        if (!gemm(JC_EPI_BIAS | JC_EPI_RES | JC_EPI_STATS, tm_f, w16 + h.l2_w.off, n, D, F, hx, hx,
                  nullptr, nullptr, stats_a, nullptr, 0, nullptr, w32 + h.l2_b.off, 0.f, s))
            return false;
    }
    if (k == 0) return true;
    // Scorer on the marker rows only (rows do not interact after the head's last attention).
    if (!launch_gather_rows(hx, stats_a, D, markers, k, xs, stats_s, s, true)) return false;
    if (!gemm(JC_EPI_LN | JC_EPI_BIAS | JC_EPI_GELU, tm_xs, w16 + P.s_lin1_w.off, k, S, D, ys,
              nullptr, stats_s, w32 + P.s_lin1_colsum.off, nullptr, nullptr, 0, nullptr,
              w32 + P.s_lin1_b.off, eps, s))
        return false;
    return launch_score(ys, S, reinterpret_cast<const __half *>(w16 + P.s_lin2_w.off), P.s_lin2_b, iota, k, logits, s, true);
}

bool Engine::enqueue_forward(uint32_t n, uint32_t k, uint32_t qtype, int fused,
                             uint16_t *d_trace, cudaStream_t s) {
    if (n == 0 || n > max_length || k > max_length || qtype >= (uint32_t)cfg.n_qtypes) {
        set_error("engine: sequence length, marker count or question type out of range");
        return false;
    }
    if (fused) {
        set_error("engine: the persistent layer kernel is not available in this build");
        return false;
    }
    const uint32_t D = cfg.d_model;
    if (!launch_embed(ids, n, reinterpret_cast<const __half *>(w16 + hw.layout.tok_emb.off), w32 + hw.layout.emb_norm.off, D,
                      cfg.norm_eps, x, nullptr, s, true))
        return false;
    for (int l = 0; l < cfg.n_layers; l++) {
        if (!encoder_layer(l, n, s)) return false;
        if (d_trace && !cuda_ok(cudaMemcpyAsync(d_trace + (size_t)l * n * D, x, (size_t)n * D * 2,
                                                cudaMemcpyDeviceToDevice, s),
                                "trace copy"))
            return false;
    }
    return head_and_scorer(n, k, qtype, s);
}

int Engine::launches_per_forward(uint32_t n, uint32_t k, int fused) const {
    (void)n;
    (void)fused;
    int c = 1 + 5 * cfg.n_layers + 1 + 5 * cfg.n_head_layers;
    if (k) c += 3;
    return c;
}

bool Engine::launch_forward(uint32_t n, uint32_t k, uint32_t qtype, int fused, cudaStream_t s) {
    GraphKey key{n, k, qtype, fused};
    auto it = graphs.find(key);
    if (it == graphs.end()) {
        cudaStream_t cap = stream;
        if (!cuda_ok(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "begin capture"))
            return false;
        const bool ok = enqueue_forward(n, k, qtype, fused, nullptr, cap);
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(cap, &graph);
        if (!ok) {
            if (graph) cudaGraphDestroy(graph);
            return false;
        }
        if (!cuda_ok(e, "end capture")) return false;
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (!cuda_ok(e, "graph instantiate")) return false;
        if ((int)graphs.size() >= GRAPH_CACHE) {
            GraphKey old = graph_lru.back();
            graph_lru.pop_back();
            cudaGraphExecDestroy(graphs[old]);
            graphs.erase(old);
        }
        it = graphs.emplace(key, exec).first;
        graph_lru.push_front(key);
    } else {
        graph_lru.remove(key);
        graph_lru.push_front(key);
    }
    return cuda_ok(cudaGraphLaunch(it->second, s), "graph launch");
}

bool Engine::check_device_error(std::string *why) {
    unsigned int code = 0;
    if (!read_device_error(&code)) {
        *why = last_error();
        return false;
    }
    if (code) {
        *why = std::string("device error: ") + device_error_name(code);
        return false;
    }
    return true;
}

}  // namespace jc
