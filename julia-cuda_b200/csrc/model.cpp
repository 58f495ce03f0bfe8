// Host-side model code: raw layout, synthetic weights and load-time preparation.
#include "model.h"

#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <thread>

namespace jc {

bool check_config(const jc_model_config &c, std::string *why) {
    auto bad = [&](const char *m) { if (why) *why = m; return false; };
    if (c.d_model <= 0 || c.d_model % 128 || c.d_model > 1024)
        return bad("d_model must be a multiple of 128 up to 1024");
    if (c.n_heads * 64 != c.d_model) return bad("n_heads must be d_model / 64");
    if (c.inter <= 0 || c.inter % 64) return bad("inter must be a positive multiple of 64");
    if (c.head_ff <= 0 || c.head_ff % 64) return bad("head_ff must be a positive multiple of 64");
    if (c.scorer_hidden <= 0 || c.scorer_hidden % 64)
        return bad("scorer_hidden must be a positive multiple of 64");
    if (c.n_layers < 1 || c.n_layers > 256) return bad("n_layers must be 1..256");
    if (c.n_head_layers < 0 || c.n_head_layers > 16) return bad("n_head_layers must be 0..16");
    if (c.vocab < 1) return bad("vocab must be positive");
    if (c.global_every < 1) return bad("global_every must be >= 1");
    if (c.window < 0) return bad("window must be >= 0");
    if (c.max_positions < 1) return bad("max_positions must be positive");
    if (c.n_qtypes < 1) return bad("n_qtypes must be positive");
    return true;
}

RawLayout raw_layout(const jc_model_config &c) {
    RawLayout o;
    size_t at = 0;
    const size_t D = c.d_model, I = c.inter, F = c.head_ff, S = c.scorer_hidden;
    auto put = [&](size_t n) {
        Span s{at, n};
        at += n;
        o.order.push_back(s);
        return s;
    };
    o.tok_emb = put((size_t)c.vocab * D);
    o.emb_norm = put(D);
    for (int l = 0; l < c.n_layers; l++) {
        o.attn_norm.push_back(put(l == 0 ? 0 : D));
        o.wqkv.push_back(put(3 * D * D));
        o.wo.push_back(put(D * D));
        o.mlp_norm.push_back(put(D));
        o.wi.push_back(put(2 * I * D));
        o.wo_mlp.push_back(put(D * I));
    }
    o.final_norm = put(D);
    o.type_emb = put((size_t)c.n_qtypes * D);
    for (int l = 0; l < c.n_head_layers; l++) {
        o.h_norm1_w.push_back(put(D));
        o.h_norm1_b.push_back(put(D));
        o.h_in_w.push_back(put(3 * D * D));
        o.h_in_b.push_back(put(3 * D));
        o.h_out_w.push_back(put(D * D));
        o.h_out_b.push_back(put(D));
        o.h_norm2_w.push_back(put(D));
        o.h_norm2_b.push_back(put(D));
        o.h_l1_w.push_back(put(F * D));
        o.h_l1_b.push_back(put(F));
        o.h_l2_w.push_back(put(D * F));
        o.h_l2_b.push_back(put(D));
    }
    o.s_norm_w = put(D);
    o.s_norm_b = put(D);
    o.s_lin1_w = put(S * D);
    o.s_lin1_b = put(S);
    o.s_lin2_w = put(S);
    o.s_lin2_b = put(1);
    o.total = at;
    return o;
}

// ---------------------------------------------------------------------------------------------
// synthetic weights: a counter-based generator (splitmix64 finaliser over the element index, two
// uniforms per element, Box-Muller), so every element is independent and the fill parallelises.

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static inline float gauss(uint64_t stream, size_t i) {
    const uint64_t r1 = mix64(stream + 0x9e3779b97f4a7c15ULL * (2 * (uint64_t)i + 1));
    const uint64_t r2 = mix64(stream + 0x9e3779b97f4a7c15ULL * (2 * (uint64_t)i + 2));
    const double u1 = ((double)(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(r2 >> 11) * (1.0 / 9007199254740992.0);
    return (float)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

template <typename F>
static void parallel_for(size_t n, F &&f) {
    unsigned th = std::thread::hardware_concurrency();
    if (th == 0) th = 1;
    if (th > 32) th = 32;
    if (n < (1u << 16)) th = 1;
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < th; t++)
        pool.emplace_back([&, t] {
            const size_t lo = n * t / th, hi = n * (t + 1) / th;
            for (size_t i = lo; i < hi; i++) f(i);
        });
    for (auto &p : pool) p.join();
}

static void fill(float *raw, Span sp, uint64_t seed, int tensor, float mean, float std) {
    if (!sp.len) return;
    const uint64_t s = mix64((seed * 0x100000001b3ULL + (uint64_t)tensor * 7919) ^ 0x5bd1e9955bd1e995ULL);
    float *dst = raw + sp.off;
    parallel_for(sp.len, [&](size_t i) { dst[i] = mean + std * gauss(s, i); });
}

void init_random(const jc_model_config &c, uint64_t seed, float *raw) {
    const RawLayout L = raw_layout(c);
    int t = 0;
    const float W = 0.02f, G = 0.05f;
    fill(raw, L.tok_emb, seed, t++, 0.f, W);
    fill(raw, L.emb_norm, seed, t++, 1.f, G);
    for (int l = 0; l < c.n_layers; l++) {
        fill(raw, L.attn_norm[l], seed, t++, 1.f, G);
        fill(raw, L.wqkv[l], seed, t++, 0.f, W);
        fill(raw, L.wo[l], seed, t++, 0.f, W);
        fill(raw, L.mlp_norm[l], seed, t++, 1.f, G);
        fill(raw, L.wi[l], seed, t++, 0.f, W);
        fill(raw, L.wo_mlp[l], seed, t++, 0.f, W);
    }
    fill(raw, L.final_norm, seed, t++, 1.f, G);
    fill(raw, L.type_emb, seed, t++, 0.f, W);
    for (int l = 0; l < c.n_head_layers; l++) {
        fill(raw, L.h_norm1_w[l], seed, t++, 1.f, G);
        fill(raw, L.h_norm1_b[l], seed, t++, 0.f, W);
        fill(raw, L.h_in_w[l], seed, t++, 0.f, W);
        fill(raw, L.h_in_b[l], seed, t++, 0.f, W);
        fill(raw, L.h_out_w[l], seed, t++, 0.f, W);
        fill(raw, L.h_out_b[l], seed, t++, 0.f, W);
        fill(raw, L.h_norm2_w[l], seed, t++, 1.f, G);
        fill(raw, L.h_norm2_b[l], seed, t++, 0.f, W);
        fill(raw, L.h_l1_w[l], seed, t++, 0.f, W);
        fill(raw, L.h_l1_b[l], seed, t++, 0.f, W);
        fill(raw, L.h_l2_w[l], seed, t++, 0.f, W);
        fill(raw, L.h_l2_b[l], seed, t++, 0.f, W);
    }
    fill(raw, L.s_norm_w, seed, t++, 1.f, G);
    fill(raw, L.s_norm_b, seed, t++, 0.f, W);
    fill(raw, L.s_lin1_w, seed, t++, 0.f, W);
    fill(raw, L.s_lin1_b, seed, t++, 0.f, W);
    fill(raw, L.s_lin2_w, seed, t++, 0.f, W);
    fill(raw, L.s_lin2_b, seed, t++, 0.f, W);
}

// ---------------------------------------------------------------------------------------------
// preparation

uint16_t f16_bits(float x) {
    __half h = __float2half_rn(x);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

float f16_value(uint16_t b) {
    __half_raw r;
    r.x = b;
    return __half2float(__half(r));
}

// src/prep.rs:22-35. The column sums come from the rounded f16 W', so mean * colsum cancels the
// mean part of x . W'^T as the GEMM computes it; summing f16 values in f64 is exact.
void fold_layernorm(const float *w, const float *gamma, uint32_t out, uint32_t k, uint16_t *w16,
                    float *colsum) {
    parallel_for(out, [&](size_t j) {
        double s = 0;
        for (uint32_t p = 0; p < k; p++) {
            const uint16_t b = f16_bits(w[j * k + p] * gamma[p]);
            w16[j * k + p] = b;
            s += (double)f16_value(b);
        }
        colsum[j] = (float)s;
    });
}

// src/prep.rs:42-59: LN(x).W^T + b = rstd (x.W'^T - mean colsum) + (b + W.beta), W.beta in f64
// from the f32 W, summed in k order.
void fold_layernorm_bias(const float *w, const float *gamma, const float *beta, const float *b,
                         uint32_t out, uint32_t k, uint16_t *w16, float *colsum, float *bias) {
    parallel_for(out, [&](size_t j) {
        double wb = 0;
        for (uint32_t p = 0; p < k; p++) wb += (double)w[j * k + p] * (double)beta[p];
        bias[j] = (float)((double)b[j] + wb);
    });
    fold_layernorm(w, gamma, out, k, w16, colsum);
}

// The GeGLU epilogue reads 64 packed columns per chunk: 32 GELU inputs, then their 32 gates.
template <typename T>
void interleave_geglu(const T *w, uint32_t n, uint32_t k, T *out) {
    const uint32_t inter = n / 2;
    for (uint32_t p = 0; p < n; p++) {
        const uint32_t t = p / 64, s = (p % 64) / 32, e = p % 32;
        const uint32_t src = t * 32 + e + (s ? inter : 0);
        std::memcpy(out + (size_t)p * k, w + (size_t)src * k, sizeof(T) * k);
    }
}
template void interleave_geglu<uint16_t>(const uint16_t *, uint32_t, uint32_t, uint16_t *);
template void interleave_geglu<float>(const float *, uint32_t, uint32_t, float *);

// src/prep.rs:106-118: inv_freq_j = 1 / theta^(2j/64) and the angles in f32.
void rope_table(float theta, uint32_t n, float *out) {
    float inv[32];
    for (int j = 0; j < 32; j++) inv[j] = 1.0f / std::pow(theta, (float)(2 * j) / 64.0f);
    for (uint32_t p = 0; p < n; p++)
        for (int j = 0; j < 32; j++) {
            const float a = (float)p * inv[j];
            out[((size_t)p * 32 + j) * 2] = std::cos(a);
            out[((size_t)p * 32 + j) * 2 + 1] = std::sin(a);
        }
}

void rope_table_gemm(const float *table, uint32_t rows, uint32_t stride, float *out) {
    for (uint32_t g = 0; g < 16; g++)
        for (uint32_t r = 0; r < stride; r++)
            for (uint32_t e = 0; e < 4; e++)
                out[((size_t)g * stride + r) * 4 + e] = r < rows ? table[(size_t)r * 64 + 4 * g + e] : 0.f;
}

namespace {
struct Arena16 {
    std::vector<uint16_t> data;
    Span push(size_t n) {
        size_t start = (data.size() + 63) / 64 * 64;  // 128 bytes
        data.resize(start + n);
        return Span{start, n};
    }
};
struct Arena32 {
    std::vector<float> data;
    Span push(size_t n) {
        size_t start = (data.size() + 31) / 32 * 32;  // 128 bytes
        data.resize(start + n);
        return Span{start, n};
    }
};
}  // namespace

bool prepare_weights(const jc_model_config &c, const float *raw, uint32_t rope_len,
                     HostWeights *out, std::string *why) {
    if (!check_config(c, why)) return false;
    const RawLayout L = raw_layout(c);
    const uint32_t D = c.d_model, I = c.inter, F = c.head_ff, S = c.scorer_hidden;
    Arena16 h;
    Arena32 f;
    PreparedLayout &P = out->layout;
    auto conv = [&](Span src) {
        Span s = h.push(src.len);
        uint16_t *dst = h.data.data() + s.off;
        const float *from = raw + src.off;
        parallel_for(src.len, [&](size_t i) { dst[i] = f16_bits(from[i]); });
        return s;
    };
    auto copy32 = [&](const float *src, size_t n) {
        Span s = f.push(n);
        std::memcpy(f.data.data() + s.off, src, n * 4);
        return s;
    };
    P.tok_emb = conv(L.tok_emb);
    P.emb_norm = copy32(raw + L.emb_norm.off, D);
    {
        std::vector<float> t((size_t)rope_len * 64);
        rope_table(c.theta_global, rope_len, t.data());
        P.rope_global = copy32(t.data(), t.size());
        rope_table(c.theta_local, rope_len, t.data());
        P.rope_local = copy32(t.data(), t.size());
    }
    std::vector<uint16_t> w16;
    std::vector<float> cs, bias;
    for (int l = 0; l < c.n_layers; l++) {
        LayerSpans ls;
        ls.global = l % c.global_every == 0;
        ls.has_ln = L.attn_norm[l].len > 0;
        if (ls.has_ln) {
            w16.resize((size_t)3 * D * D);
            cs.resize(3 * D);
            fold_layernorm(raw + L.wqkv[l].off, raw + L.attn_norm[l].off, 3 * D, D, w16.data(),
                           cs.data());
            ls.wqkv = h.push(w16.size());
            std::memcpy(h.data.data() + ls.wqkv.off, w16.data(), w16.size() * 2);
            ls.qkv_colsum = copy32(cs.data(), cs.size());
        } else {
            ls.wqkv = conv(L.wqkv[l]);
        }
        ls.wo = conv(L.wo[l]);
        w16.resize((size_t)2 * I * D);
        cs.resize(2 * I);
        fold_layernorm(raw + L.wi[l].off, raw + L.mlp_norm[l].off, 2 * I, D, w16.data(), cs.data());
        ls.wi = h.push(w16.size());
        interleave_geglu(w16.data(), 2 * I, D, h.data.data() + ls.wi.off);
        ls.wi_colsum = f.push(2 * I);
        interleave_geglu(cs.data(), 2 * I, 1, f.data.data() + ls.wi_colsum.off);
        ls.wo_mlp = conv(L.wo_mlp[l]);
        P.layers.push_back(ls);
    }
    P.final_norm = copy32(raw + L.final_norm.off, D);
    P.type_emb = copy32(raw + L.type_emb.off, (size_t)c.n_qtypes * D);
    for (int l = 0; l < c.n_head_layers; l++) {
        HeadSpans hs;
        w16.resize((size_t)3 * D * D);
        cs.resize(3 * D);
        bias.resize(3 * D);
        fold_layernorm_bias(raw + L.h_in_w[l].off, raw + L.h_norm1_w[l].off,
                            raw + L.h_norm1_b[l].off, raw + L.h_in_b[l].off, 3 * D, D, w16.data(),
                            cs.data(), bias.data());
        hs.in_w = h.push(w16.size());
        std::memcpy(h.data.data() + hs.in_w.off, w16.data(), w16.size() * 2);
        hs.in_colsum = copy32(cs.data(), 3 * D);
        hs.in_b = copy32(bias.data(), 3 * D);
        hs.out_w = conv(L.h_out_w[l]);
        hs.out_b = copy32(raw + L.h_out_b[l].off, D);
        w16.resize((size_t)F * D);
        cs.resize(F);
        bias.resize(F);
        fold_layernorm_bias(raw + L.h_l1_w[l].off, raw + L.h_norm2_w[l].off,
                            raw + L.h_norm2_b[l].off, raw + L.h_l1_b[l].off, F, D, w16.data(),
                            cs.data(), bias.data());
        hs.l1_w = h.push(w16.size());
        std::memcpy(h.data.data() + hs.l1_w.off, w16.data(), w16.size() * 2);
        hs.l1_colsum = copy32(cs.data(), F);
        hs.l1_b = copy32(bias.data(), F);
        hs.l2_w = conv(L.h_l2_w[l]);
        hs.l2_b = copy32(raw + L.h_l2_b[l].off, D);
        P.head.push_back(hs);
    }
    w16.resize((size_t)S * D);
    cs.resize(S);
    bias.resize(S);
    fold_layernorm_bias(raw + L.s_lin1_w.off, raw + L.s_norm_w.off, raw + L.s_norm_b.off,
                        raw + L.s_lin1_b.off, S, D, w16.data(), cs.data(), bias.data());
    P.s_lin1_w = h.push(w16.size());
    std::memcpy(h.data.data() + P.s_lin1_w.off, w16.data(), w16.size() * 2);
    P.s_lin1_colsum = copy32(cs.data(), S);
    P.s_lin1_b = copy32(bias.data(), S);
    P.s_lin2_w = conv(L.s_lin2_w);
    P.s_lin2_b = raw[L.s_lin2_b.off];
    out->f16 = std::move(h.data);
    out->f32 = std::move(f.data);
    return true;
}

}  // namespace jc
