// The model on the host: the raw (checkpoint-like) f32 format, seeded synthetic weights, and the
// load-time preparation into the layouts the kernels read (the reference's src/weights.rs and
// src/prep.rs).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/julia_cuda.h"

namespace jc {

struct Span {
    size_t off = 0, len = 0;
};

// Offsets of every raw tensor (in the order julia_cuda.h documents).
struct RawLayout {
    Span tok_emb, emb_norm;
    std::vector<Span> attn_norm, wqkv, wo, mlp_norm, wi, wo_mlp;
    Span final_norm, type_emb;
    std::vector<Span> h_norm1_w, h_norm1_b, h_in_w, h_in_b, h_out_w, h_out_b, h_norm2_w,
        h_norm2_b, h_l1_w, h_l1_b, h_l2_w, h_l2_b;
    Span s_norm_w, s_norm_b, s_lin1_w, s_lin1_b, s_lin2_w, s_lin2_b;
    size_t total = 0;
    std::vector<Span> order;  // every span in raw order
};

bool check_config(const jc_model_config &c, std::string *why);
RawLayout raw_layout(const jc_model_config &c);
void init_random(const jc_model_config &c, uint64_t seed, float *raw);

// host preparation (bit patterns for f16)
uint16_t f16_bits(float x);
float f16_value(uint16_t h);
void fold_layernorm(const float *w, const float *gamma, uint32_t out, uint32_t k, uint16_t *w16,
                    float *colsum);
void fold_layernorm_bias(const float *w, const float *gamma, const float *beta, const float *b,
                         uint32_t out, uint32_t k, uint16_t *w16, float *colsum, float *bias);
template <typename T>
void interleave_geglu(const T *w, uint32_t n, uint32_t k, T *out);
void rope_table(float theta, uint32_t n, float *out);
// The GEMM epilogue's layout of a RoPE table: float4 out[16][stride] with out[g][r] = (cos, sin) of
// pairs 2g and 2g + 1 of row r, from the natural [rows][32][2] table (rows <= stride).
void rope_table_gemm(const float *table, uint32_t rows, uint32_t stride, float *out);

// The prepared weights: f16 matrices in one arena and f32 vectors in another, every span
// 128-byte aligned (the reference's two-arena layout, src/weights.rs:19-140).
struct LayerSpans {
    Span wqkv, qkv_colsum, wo, wi, wi_colsum, wo_mlp;
    bool global = false, has_ln = false;
};
struct HeadSpans {
    Span in_w, in_colsum, in_b, out_w, out_b, l1_w, l1_colsum, l1_b, l2_w, l2_b;
};
struct PreparedLayout {
    Span tok_emb, emb_norm, rope_global, rope_local, final_norm, type_emb;
    std::vector<LayerSpans> layers;
    std::vector<HeadSpans> head;
    Span s_lin1_w, s_lin1_colsum, s_lin1_b, s_lin2_w;
    float s_lin2_b = 0.f;
};
struct HostWeights {
    PreparedLayout layout;
    std::vector<uint16_t> f16;
    std::vector<float> f32;
};

// max_positions of the RoPE tables = rope_len.
bool prepare_weights(const jc_model_config &c, const float *raw, uint32_t rope_len,
                     HostWeights *out, std::string *why);

}  // namespace jc
