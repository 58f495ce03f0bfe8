/*
 * CPU ORACLE for the julia-cuda encoder hot path. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
 * load this library, and only as the checker or as the timed CPU baseline; the product path
 * (julia-cuda_b200/) never calls it.
 *
 * What it restates (the reference is Rust, arnu515/julia-cuda, and its f32 CPU path lives in the
 * un-vendored crate julia-rs @ git 6006d2bcdb3533840c530aee99cd8cb9b6aab6a9, Cargo.lock:218-220):
 *   - or_forward_f32: the f32 model as the reference's checks drive julia-rs
 *     (src/check.rs:177-224 `trace`, :484-548 `head_trace`), LayerNorms in f64.
 *   - or_emu_*: the f16-storage / f32-accumulation arithmetic of the GPU kernels, restated from
 *     the reference's host emulation (src/check.rs:64-123 emulate_embed/emulate_gemm, :879-1076
 *     HostEncoder, src/prep.rs:166-186 folded_gpu), in the logical (unpermuted) layouts.
 *   - prep: fold_layernorm (src/prep.rs:22-35), fold_layernorm_bias (:42-59), rope_table
 *     (:106-118), and the reference's own permute_rope (:88-101) / interleave_geglu (:67-77)
 *     layouts so their known-answer tests can be restated.
 *   - the reference's layer-kernel plan model: phase_cost / gemm_plan (src/forward.rs:761-806).
 *
 * Parity pinning: the prep transforms and the plan model are pinned by the reference's own
 * known-answer tests (src/prep.rs:252-327, src/forward.rs:815-823), restated in tests/. The forward
 * numerics cannot be pinned to julia-rs (crate and checkpoint absent); the f32 forward is pinned to
 * implementations written outside this project on the same checkpoint (transformers'
 * ModernBertModel for the encoder, torch.nn.TransformerEncoderLayer and nn.LayerNorm / Linear /
 * GELU for the head and scorer, tests/test_hf_modernbert.py), to an independent torch-CPU f32
 * restatement in tests/, and the emulation to the f32 forward within the reference's tolerance
 * design (src/check.rs:382-402).
 */
#ifndef JC_ORACLE_H
#define JC_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#define OR_MAX_LAYERS 64
#define OR_MAX_HEAD 4

typedef struct {
    int32_t d_model;        /* D: hidden width (384 in the reference, 768 in the benchmark) */
    int32_t n_heads;        /* D / 64 */
    int32_t inter;          /* GeGLU intermediate (1152) */
    int32_t n_layers;       /* encoder layers (22) */
    int32_t vocab;          /* 50368 */
    int32_t head_ff;        /* head linear1 width */
    int32_t scorer_hidden;  /* scorer lin1 width (D in the reference, 384 in the benchmark) */
    int32_t n_head_layers;  /* 2 */
    int32_t global_every;   /* layer l is global when l % global_every == 0 */
    int32_t window;         /* sliding-window reach: |q - k| <= window (local_window / 2 = 64) */
    int32_t max_positions;  /* RoPE table length */
    int32_t n_qtypes;       /* type embeddings (3: choice, score, noul) */
    float norm_eps;         /* encoder LayerNorm eps */
    float head_eps;         /* head / scorer LayerNorm eps (nn.LayerNorm default 1e-5) */
    float theta_global;     /* 160000 */
    float theta_local;      /* 10000 */
} or_config;

typedef struct { size_t off, len; } or_span;

/* The raw (checkpoint-like) f32 model: every tensor in one buffer, packed in this order. */
typedef struct {
    or_span tok_emb, emb_norm;
    or_span attn_norm[OR_MAX_LAYERS], wqkv[OR_MAX_LAYERS], wo[OR_MAX_LAYERS];
    or_span mlp_norm[OR_MAX_LAYERS], wi[OR_MAX_LAYERS], wo_mlp[OR_MAX_LAYERS];
    or_span final_norm, type_emb;
    or_span h_norm1_w[OR_MAX_HEAD], h_norm1_b[OR_MAX_HEAD], h_in_w[OR_MAX_HEAD], h_in_b[OR_MAX_HEAD];
    or_span h_out_w[OR_MAX_HEAD], h_out_b[OR_MAX_HEAD], h_norm2_w[OR_MAX_HEAD], h_norm2_b[OR_MAX_HEAD];
    or_span h_l1_w[OR_MAX_HEAD], h_l1_b[OR_MAX_HEAD], h_l2_w[OR_MAX_HEAD], h_l2_b[OR_MAX_HEAD];
    or_span s_norm_w, s_norm_b, s_lin1_w, s_lin1_b, s_lin2_w, s_lin2_b;
    size_t total;
} or_layout;

#ifdef __cplusplus
extern "C" {
#endif

int or_layout_of(const or_config *c, or_layout *out);
size_t or_raw_size(const or_config *c);
/* Seeded random init: matrices / embeddings / biases / type embeddings N(0, 0.02), LayerNorm
 * gammas 1 + N(0, 0.05), LayerNorm betas N(0, 0.02). */
void or_init_random(const or_config *c, uint64_t seed, float *raw);
/* Seeded normal fill (splitmix64 + Box-Muller), for synthetic activations. */
void or_fill_normal(float *dst, size_t n, uint64_t seed, float mean, float std);

/* f32 model: logits for the marker rows. If trace_x is not NULL it receives the residual stream
 * after each encoder layer ([n_layers][n][D]). Returns 0 or -1 on bad arguments. */
int or_forward_f32(const or_config *c, const float *raw, const uint32_t *ids, int n,
                   const uint32_t *markers, int n_markers, int qtype, float *logits,
                   float *trace_x);
/* The same with the head on rows [0, head_rows) only (0: all rows): the final LayerNorm, the
 * head layers (their attention over those rows) and the marker rows; markers must be below
 * head_rows. BASELINE config 4's long-context request (1024 tokens, head on 512 rows). */
int or_forward_f32_head(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x);
/* The same with the head traced, as the reference's --check traces it from the encoder output
 * (src/check.rs:484-548 head_trace, :564-596 head): head_trace (if not NULL) receives the head's
 * stream [n_head_layers + 1][nh][D] (its input after the final LayerNorm and type embedding, then
 * after each head layer; nh = the head's rows), scorer_trace (if not NULL) the scorer's hidden
 * layer after GELU for each marker [n_markers][scorer_hidden]. */
int or_forward_f32_full(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, float *head_trace, float *scorer_trace);

/* The f16 emulation of the GPU path (same folds, roundings and statistics as the kernels) over the
 * same raw weights; same outputs as or_forward_f32. trace_x gets the f16 residual stream after each
 * layer as f32. bugs: bit 0 naive GeGLU halves swapped, bit 1 no RoPE, bit 2 no window (the
 * reference's negative tests, src/check.rs:879-895). */
int or_forward_emu(const or_config *c, const float *raw, const uint32_t *ids, int n,
                   const uint32_t *markers, int n_markers, int qtype, float *logits,
                   float *trace_x, int bugs);
int or_forward_emu_head(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, int bugs);
/* With the head and scorer traced as or_forward_f32_full (f16 values as f32). */
int or_forward_emu_full(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, float *head_trace, float *scorer_trace,
                        int bugs);

/* ---- f16-arithmetic emulation of single kernels (inputs/outputs are f16 bit patterns) ---- */
/* Epilogue flags, as the GEMM family's. */
enum { OR_RES = 1, OR_GEGLU = 2, OR_LN = 4, OR_STATS = 8, OR_ROPE = 16, OR_BIAS = 32,
       OR_RELU = 64, OR_GELU = 128 };
/* c = epilogue(a . w^T) in LOGICAL layout: a [m,k] f16, w [n,k] f16 (for GEGLU, rows [0,n/2) are
 * the GELU inputs and [n/2,n) the gates, c is [m, n/2]); ROPE rotates dims (i, i+32) of every
 * 64-wide head in the first two thirds of c using rope [pos][32][2]; stats_out gets += row sums of
 * the stored f16 outputs. */
void or_emu_gemm(int epi, const uint16_t *a, const uint16_t *w, uint16_t *c, int m, int n, int k,
                 const float *stats_in, const float *colsum, float eps, const float *rope,
                 const float *bias, float *stats_out);
/* o = attention(qkv) per head (H heads of 64), P rounded to f16, keys |q-k| <= window (0: all). */
void or_emu_attention(const uint16_t *qkv, uint16_t *o, int n, int heads, int window);
/* The same attention in f32 from f32 q/k/v (no f16 rounding). */
void or_attention_f32(const float *qkv, float *o, int n, int heads, int window);
void or_emu_embed(const uint16_t *table, const float *gamma, const uint32_t *ids, int n, int d,
                  float eps, uint16_t *x);
void or_emu_norm_add(const uint16_t *x, const float *gamma, const float *add, int n, int d,
                     float eps, uint16_t *out, float *stats);
void or_emu_score(const uint16_t *y, const uint16_t *w, float b, const uint32_t *markers, int k,
                  int d, float *logits);
void or_row_stats(const uint16_t *x, int n, int d, float *stats);

/* ---- weight preparation (reference algorithms) ---- */
/* W' = f16(w * gamma) (w [out,k] f32), colsum[j] = sum_k W'[j,k] in f64 of the rounded values. */
void or_fold_layernorm(const float *w, const float *gamma, int out, int k, uint16_t *w16,
                       float *colsum);
/* Also bias' = b + W . beta (f64 from the f32 W). */
void or_fold_layernorm_bias(const float *w, const float *gamma, const float *beta, const float *b,
                            int out, int k, uint16_t *w16, float *colsum, float *bias);
/* RoPE (cos, sin) table [n][32][2], f32 as the reference computes it. */
void or_rope_table(float theta, int n, float *out);
/* The reference's mma.sync-fragment layouts (row index maps), for its known-answer tests. */
void or_ref_permute_rope_rows(int n, int32_t *src_of_row);
void or_ref_interleave_geglu_rows(int n, int32_t *src_of_row);
/* The reference's layer-kernel cost model and per-GEMM plan (fitted to a 2080 Ti). */
double or_ref_phase_cost(int n, int cols, int k, int bm, int z, int sms, int per_sm);
void or_ref_gemm_plan(int n, int cols, int k, int sms, int per_sm, int *bm, int *z);

/* f16 helpers (round to nearest even). */
uint16_t or_f16_from_f32(float x);
float or_f32_from_f16(uint16_t h);
void or_f16_round_array(const float *src, uint16_t *dst, size_t n);

/* A&S 7.1.26 erf-based GELU, in f64 (the kernels' formula). */
float or_gelu(float x);

int or_num_threads(void);
/* Threads the oracle's parallel loops use from now on (OpenMP; launchers such as torchrun set
 * OMP_NUM_THREADS=1 for every rank). */
void or_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
