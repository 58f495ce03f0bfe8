// jc_layer: one encoder layer on the persistent kernel, over device buffers the caller owns -- the
// kernel-level boundary of the reference's persistent `layer` kernel (kernels/src/main.rs:579-606,
// launched by src/forward.rs:226-359), which the engine's layer-fused mode (julia_cuda_run with
// layer_fused = 1) runs once per layer.
//
// The five phases are those of the engine's layer (engine.cpp, build_steps_flat): qkv (LayerNorm
// folded unless qkv_colsum is NULL, RoPE; clears stats_attn), attention (global, or keys within
// `window`), wo (x += o Wo^T, row statistics into stats_attn), wi (LayerNorm folded, GeGLU into
// mbuf; clears stats_mlp) and wo_mlp (x += m Wo_mlp^T, row statistics into stats_mlp). The tile
// plan (plan_flow) and the launch are the engine's; the phase descriptors, tensor maps and
// completion counters live in a per-device scratch allocated on first use and grown with the row
// count, so calls on one device must not overlap in time (one stream, or synchronised by the
// caller), as one engine serves one thread in the reference.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/julia_cuda.h"
#include "jc_internal.h"
#include "params.h"

namespace {

constexpr uint32_t LAYER_PHASES = 5;
constexpr uint32_t LAYER_MAPS = 7;  // A: x, o, m; W: wqkv, wo, wi, wo_mlp

struct LayerScratch {
    jc::PhaseDesc *descs = nullptr;
    CUtensorMap *maps = nullptr;
    uint32_t *ctr = nullptr;
    uint32_t blocks = 0;  // row blocks the counters cover
    uint32_t grid = 0;    // the persistent kernel's CTAs on this device
};

std::mutex g_layer_mu;
LayerScratch g_layer[64];

bool fail(const std::string &msg) {
    jc::set_error("layer: " + msg);
    return false;
}

bool cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    return fail(std::string(what) + ": " + cudaGetErrorString(e));
}

// The device's scratch, with counters for at least `blocks` row blocks.
LayerScratch *scratch(int dev, uint32_t blocks) {
    if (dev < 0 || dev >= 64) {
        fail("device index out of range");
        return nullptr;
    }
    LayerScratch &s = g_layer[dev];
    if (!s.descs) {
        if (!cuda(cudaMalloc(&s.descs, LAYER_PHASES * sizeof(jc::PhaseDesc)), "cudaMalloc") ||
            !cuda(cudaMalloc(&s.maps, LAYER_MAPS * sizeof(CUtensorMap)), "cudaMalloc"))
            return nullptr;
        int sms = 0;
        if (!cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "sm count"))
            return nullptr;
        s.grid = (uint32_t)(sms * jc::persist_blocks_per_sm());
        if (s.grid == 0) {
            fail("the persistent kernel cannot be resident on this GPU");
            return nullptr;
        }
    }
    if (s.blocks < blocks) {
        // Grown in powers of two; the counters are zero between launches (the kernel's last CTA
        // clears them), so a fresh allocation starts zeroed.
        uint32_t b = s.blocks ? s.blocks : 8;
        while (b < blocks) b *= 2;
        if (s.ctr && !cuda(cudaDeviceSynchronize(), "sync")) return nullptr;
        if (s.ctr) cudaFree(s.ctr);
        s.ctr = nullptr;
        s.blocks = 0;
        const size_t words = jc::flow_counter_words(LAYER_PHASES, b);
        if (!cuda(cudaMalloc(&s.ctr, words * 4), "cudaMalloc") ||
            !cuda(cudaMemset(s.ctr, 0, words * 4), "cudaMemset"))
            return nullptr;
        s.blocks = b;
    }
    return &s;
}

jc::PhaseDesc gemm_phase(uint32_t epi, __half *c, const __half *res, const float *stats_in,
                         const float *colsum, float *stats_out, float *zero, uint32_t zero_len,
                         const float *rope, uint32_t rope_stride, uint32_t m, uint32_t n,
                         uint32_t k, float eps) {
    jc::PhaseDesc d{};
    d.kind = jc::PH_GEMM;
    d.epi = epi;
    jc::GemmParams &g = d.g;
    g.c = c;
    g.res = res;
    g.stats_in = stats_in;
    g.colsum = colsum;
    g.stats_out = stats_out;
    g.zero = zero;
    g.zero_len = zero_len;
    g.rope = rope;
    g.rope_stride = rope_stride;
    g.m = m;
    g.n = n;
    g.k = k;
    g.eps = eps;
    return d;
}

}  // namespace

extern "C" int jc_layer(uint16_t *x, uint16_t *qkv, uint16_t *o, uint16_t *mbuf, float *stats_attn,
                        float *stats_mlp, const uint16_t *wqkv, const float *qkv_colsum,
                        const float *rope, uint32_t rope_stride, const uint16_t *wo,
                        const uint16_t *wi, const float *wi_colsum, const uint16_t *wo_mlp,
                        uint32_t m, uint32_t d_model, uint32_t heads, uint32_t inter, float eps,
                        uint32_t window, void *stream) {
    try {
        if (!x || !qkv || !o || !mbuf || !stats_attn || !stats_mlp || !wqkv || !rope || !wo ||
            !wi || !wi_colsum || !wo_mlp)
            return fail("a null buffer (only qkv_colsum may be NULL: no LayerNorm before qkv)"), -1;
        if (m == 0 || heads == 0 || d_model != heads * 64 || inter == 0 || inter % 64)
            return fail("rows must be positive, d_model = 64 x heads and inter a multiple of 64"), -1;
        if (rope_stride == 0) rope_stride = m;
        if (rope_stride < m) return fail("the RoPE table has fewer rows than the layer"), -1;
        if ((reinterpret_cast<uintptr_t>(stats_attn) | reinterpret_cast<uintptr_t>(stats_mlp)) & 7)
            return fail("the statistics buffers must be 8-byte aligned"), -1;
        int dev = 0;
        if (!cuda(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
        const uint32_t D = d_model, I = inter;
        const uint32_t blocks = (m + jc::FLOW_BLOCK - 1) / jc::FLOW_BLOCK;
        std::lock_guard<std::mutex> lock(g_layer_mu);
        LayerScratch *S = scratch(dev, blocks);
        if (!S) return -1;
        auto h = [](uint16_t *p) { return reinterpret_cast<__half *>(p); };
        std::vector<jc::PhaseDesc> d(LAYER_PHASES);
        d[0] = gemm_phase(qkv_colsum ? (JC_EPI_LN | JC_EPI_ROPE) : JC_EPI_ROPE, h(qkv), nullptr,
                          qkv_colsum ? stats_mlp : nullptr, qkv_colsum, nullptr, stats_attn, 2 * m,
                          rope, rope_stride, m, 3 * D, D, eps);
        d[1].kind = jc::PH_ATTN;
        d[1].a = jc::AttnParams{h(qkv), h(o), nullptr, nullptr, m, heads, window, nullptr, nullptr};
        d[2] = gemm_phase(JC_EPI_RES | JC_EPI_STATS, h(x), h(x), nullptr, nullptr, stats_attn,
                          nullptr, 0, nullptr, 0, m, D, D, 0.f);
        d[3] = gemm_phase(JC_EPI_LN | JC_EPI_GEGLU, h(mbuf), nullptr, stats_attn, wi_colsum, nullptr,
                          stats_mlp, 2 * m, nullptr, 0, m, 2 * I, D, eps);
        d[4] = gemm_phase(JC_EPI_RES | JC_EPI_STATS, h(x), h(x), nullptr, nullptr, stats_mlp,
                          nullptr, 0, nullptr, 0, m, D, I, 0.f);
        const uint32_t total = jc::plan_flow(d.data(), LAYER_PHASES, S->grid);
        // Tensor maps: the activations in 128-row boxes, the weights in boxes as tall as the tile
        // width the plan gave each GEMM phase.
        CUtensorMap hm[LAYER_MAPS];
        const void *w_of[4] = {wqkv, wo, wi, wo_mlp};
        const uint32_t w_rows[4] = {3 * D, D, 2 * I, D}, w_cols[4] = {D, D, D, I};
        const uint32_t gemm_phase_of[4] = {0, 2, 3, 4};
        if (!jc::make_tmap_f16(&hm[0], x, m, D, jc::FLOW_BLOCK) ||
            !jc::make_tmap_f16(&hm[1], o, m, D, jc::FLOW_BLOCK) ||
            !jc::make_tmap_f16(&hm[2], mbuf, m, I, jc::FLOW_BLOCK))
            return -1;
        for (int i = 0; i < 4; i++)
            if (!jc::make_tmap_f16(&hm[3 + i], w_of[i], w_rows[i], w_cols[i], d[gemm_phase_of[i]].bn))
                return -1;
        const uint32_t a_of[4] = {0, 1, 0, 2};  // qkv and wi read x, wo reads o, wo_mlp reads m
        for (int i = 0; i < 4; i++) {
            jc::GemmParams &g = d[gemm_phase_of[i]].g;
            g.map_a = S->maps + a_of[i];
            g.map_w = S->maps + 3 + i;
        }
        cudaStream_t s = (cudaStream_t)stream;
        // Both uploads are from pageable memory: staged before the calls return.
        if (!cuda(cudaMemcpyAsync(S->maps, hm, sizeof(hm), cudaMemcpyHostToDevice, s), "map upload") ||
            !cuda(cudaMemcpyAsync(S->descs, d.data(), LAYER_PHASES * sizeof(jc::PhaseDesc),
                                  cudaMemcpyHostToDevice, s),
                  "phase upload"))
            return -1;
        return jc::launch_persist(S->descs, LAYER_PHASES, total, S->ctr, S->blocks, S->grid,
                                  2000000000ull, s, nullptr)
                   ? 0
                   : -1;
    } catch (const std::exception &ex) {
        jc::set_error(std::string("layer: exception: ") + ex.what());
    } catch (...) {
        jc::set_error("layer: unknown exception");
    }
    return -1;
}
