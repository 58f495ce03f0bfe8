/*
 * julia-cuda-b200: the julia-cuda encoder hot path (ModernBERT-style encoder, 2-layer head and
 * scorer of Julia-1) on NVIDIA B200 (sm_100a). C ABI of libjulia_cuda.so.
 *
 * Conventions (as the reference's src/capi.rs:4-6, 23-54): functions returning a pointer give NULL
 * on failure and those returning an int give -1; the message goes to `err` (err_len bytes,
 * NUL-terminated, truncated) when the function takes one, else to jc_last_error(). Nothing throws
 * across the boundary. The caller owns every array. An engine must not be used by two threads at
 * once (src/capi.rs:116); use one engine per GPU for several GPUs.
 *
 * f16 values are passed as uint16_t bit patterns. "Device" pointers are CUDA device memory of the
 * current device; `stream` is a cudaStream_t (NULL: the legacy default stream).
 */
#ifndef JULIA_CUDA_H
#define JULIA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct JcEngine JcEngine;

/* The model's shape: the fields of julia-rs's ModelConfig the reference reads
 * (src/checkpoint.rs:29; hidden, intermediate, n_layers, norm_eps, local_window/2, max_positions,
 * rope_theta_global/local, vocab, head_ff) plus the head/scorer widths. */
typedef struct jc_model_config {
    int32_t d_model;       /* hidden width, a multiple of 128 up to 1024 */
    int32_t n_heads;       /* d_model / 64 */
    int32_t inter;         /* GeGLU intermediate width, a multiple of 64 */
    int32_t n_layers;      /* encoder layers */
    int32_t vocab;
    int32_t head_ff;       /* head linear1 width, a multiple of 64 */
    int32_t scorer_hidden; /* scorer lin1 width, a multiple of 64 */
    int32_t n_head_layers;
    int32_t global_every;  /* layer l uses global attention when l % global_every == 0 */
    int32_t window;        /* sliding-window reach: keys with |q - k| <= window */
    int32_t max_positions; /* RoPE table length (longest sequence) */
    int32_t n_qtypes;      /* type embeddings: 0 choice, 1 score, 2 noul */
    float norm_eps;        /* encoder LayerNorm eps */
    float head_eps;        /* head and scorer LayerNorm eps */
    float theta_global;    /* RoPE base of the global layers */
    float theta_local;     /* RoPE base of the sliding-window layers */
} jc_model_config;

/* ============================ the reference's C ABI (src/capi.rs) ============================ */

/* The kernel tier this library was built for ("sm_100a"), static. Replaces src/capi.rs:56-62. */
const char *julia_cuda_tier(void);

/* Opens a checkpoint directory and uploads it to GPU 0 (src/capi.rs:64-85). The reference's
 * layout (src/checkpoint.rs:27-62): dir/model.safetensors + dir/encoder/config.json (the
 * ModernBERT encoder's Hugging Face config) + dir/julia_config.json (the head and scorer), read as
 * julia_cuda_read_checkpoint documents; or, when there is no model.safetensors, the raw model
 * format below from dir/jc_config.bin + dir/jc_weights.f32 (julia_cuda_save_raw). `max_length` 0
 * means the model's max_positions. */
JcEngine *julia_cuda_load(const char *dir, size_t max_length, char *err, size_t err_len);

/* Frees an engine (NULL is fine). Replaces src/capi.rs:87-96. */
void julia_cuda_free(JcEngine *engine);

/* The GPU's name into buf (len bytes, NUL-terminated). Replaces src/capi.rs:98-106. */
void julia_cuda_device(const JcEngine *engine, char *buf, size_t len);

/* Runs b sequences back to back: sequence i is lens[i] token ids (concatenated in ids) with
 * n_markers[i] marker positions (concatenated in markers) and question type qtypes[i]. Writes each
 * sequence's logits (one per marker, concatenated) and its GPU time in ms (embed to logits) into
 * gpu_ms[i]. layer_fused: 0 runs one kernel per step (the reference's per-step kernels), 1 one
 * persistent launch per encoder layer (the reference's layer kernel), 2 one persistent launch for
 * the whole model, embed to logits.
 * Returns 0, or -1 with the error in err (also for non-finite logits and device-side timeouts).
 * Replaces src/capi.rs:108-190. */
int julia_cuda_run(const JcEngine *engine, size_t b, const uint32_t *ids, const size_t *lens,
                   const uint32_t *markers, const size_t *n_markers, const uint32_t *qtypes,
                   int layer_fused, float *logits, float *gpu_ms, char *err, size_t err_len);

/* ================================ additions to the reference ================================ */

/* The benchmark model: hidden 768, 12 heads, GeGLU 1152, 22 layers, vocab 50368, head_ff 2048,
 * scorer 768 -> 384 -> 1, global every 3rd layer, window 64, theta 160000 / 10000. */
void julia_cuda_default_config(jc_model_config *cfg);

/* The raw model format: every tensor f32, [out, in] matrices, packed in this order:
 * tok_embeddings [vocab, D], emb_norm [D]; per layer: attn_norm [D] (absent in layer 0),
 * Wqkv [3D, D], Wo [D, D], mlp_norm [D], Wi [2I, D] (GELU inputs, then gates), Wo_mlp [D, I];
 * final_norm [D], type_emb [n_qtypes, D]; per head layer: norm1 w, b [D], in_proj w [3D, D], b [3D],
 * out_proj w [D, D], b [D], norm2 w, b [D], linear1 w [F, D], b [F], linear2 w [D, F], b [D];
 * scorer norm w, b [D], lin1 w [S, D], b [S], lin2 w [1, S], b [1]. */
size_t julia_cuda_raw_size(const jc_model_config *cfg);
/* The offset of every tensor above, in order (cap entries at most); returns the count or -1. */
int julia_cuda_raw_offsets(const jc_model_config *cfg, size_t *offsets, size_t cap);
/* Seeded synthetic weights in the raw format: matrices, embeddings, biases, betas and type
 * embeddings N(0, 0.02); LayerNorm gammas 1 + N(0, 0.05). */
void julia_cuda_init_random(const jc_model_config *cfg, uint64_t seed, float *raw);
/* Writes cfg + raw to dir (jc_config.bin, jc_weights.f32) for julia_cuda_load. */
int julia_cuda_save_raw(const char *dir, const jc_model_config *cfg, const float *raw,
                        char *err, size_t err_len);

/* Reads a checkpoint directory (model.safetensors + encoder/config.json + julia_config.json) on the
 * host into *cfg and the raw format (raw_cap floats at raw; raw NULL: only *cfg and *raw_len).
 * Tensors are F32, F16 or BF16, named as the public layouts they come from: the encoder as Hugging
 * Face ModernBERT (`<prefix>embeddings.tok_embeddings.weight`, `<prefix>embeddings.norm.weight`,
 * `<prefix>layers.{i}.attn_norm.weight` (i > 0), `.attn.Wqkv.weight`, `.attn.Wo.weight`,
 * `.mlp_norm.weight`, `.mlp.Wi.weight` (GELU inputs, then gates), `.mlp.Wo.weight`,
 * `<prefix>final_norm.weight`; the prefix "model.", "encoder.model.", "encoder." or none, found by
 * probing), the head layers as torch.nn.TransformerEncoderLayer (`head.layers.{i}.norm1.weight`,
 * `.norm1.bias`, `.self_attn.in_proj_weight`, `.self_attn.in_proj_bias`,
 * `.self_attn.out_proj.weight`, `.self_attn.out_proj.bias`, `.norm2.weight`, `.norm2.bias`,
 * `.linear1.weight`, `.linear1.bias`, `.linear2.weight`, `.linear2.bias`), `type_emb.weight`
 * [n_qtypes, D] and `scorer.{norm,lin1,lin2}.{weight,bias}`. The reference reads the head and
 * scorer names through julia-rs (not available here), so an optional dir/jc_names.json overrides
 * any of them: {"encoder_prefix": "...", "names": {"<name above, encoder names without the
 * prefix>": "<name in the file>"}}. encoder/config.json gives hidden_size, intermediate_size,
 * num_hidden_layers, vocab_size (required), num_attention_heads, norm_eps, local_attention (the
 * window's full span), global_attn_every_n_layers, max_position_embeddings, global_rope_theta and
 * local_rope_theta; julia_config.json (optional) head_layers, head_ff, scorer_hidden, n_qtypes and
 * head_eps, each otherwise taken from the tensors' shapes (or the benchmark model's default).
 * Every shape is checked. Returns 0, or -1 with the reason. No counterpart in the reference's C
 * ABI (its Engine::load does this internally, src/engine.rs:118-150). */
int julia_cuda_read_checkpoint(const char *dir, jc_model_config *cfg, float *raw, size_t raw_cap,
                               size_t *raw_len, char *err, size_t err_len);
/* Writes cfg + raw as such a directory under the default names (dtype 0 F32, 1 F16, 2 BF16). */
int julia_cuda_save_checkpoint(const char *dir, const jc_model_config *cfg, const float *raw,
                               int dtype, char *err, size_t err_len);
/* The load-time preparation alone, on the host (src/weights.rs:143-238, src/prep.rs): the f16
 * arena (bit patterns) and the f32 arena an engine of max_length rows (0: max_positions) uploads.
 * *f16_len / *f32_len receive their sizes; f16 / f32 may be NULL to ask only for them. */
int julia_cuda_prepare_host(const jc_model_config *cfg, const float *raw, size_t raw_len,
                            size_t max_length, uint16_t *f16, size_t f16_cap, float *f32,
                            size_t f32_cap, size_t *f16_len, size_t *f32_len, char *err,
                            size_t err_len);

/* Builds an engine on GPU `device` from raw weights (prepared on the host: LayerNorm folds,
 * GeGLU interleave, f16 conversion, RoPE tables), buffers for sequences up to max_length. */
JcEngine *julia_cuda_load_raw(const jc_model_config *cfg, const float *raw, size_t raw_len,
                              size_t max_length, int device, char *err, size_t err_len);
JcEngine *julia_cuda_load_random(const jc_model_config *cfg, uint64_t seed, size_t max_length,
                                 int device, char *err, size_t err_len);

/* One sequence with inputs already on the engine's device: d_ids [n], d_markers [n_markers];
 * writes d_logits [n_markers]. Queued on `stream` (NULL: the legacy default stream), not waited
 * for.
 * d_trace, if not NULL, receives the residual stream (f16) after every encoder layer,
 * [n_layers][n][D] (slower: no CUDA graph). Returns 0 or -1. */
int julia_cuda_forward_device(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                              const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                              int layer_fused, float *d_logits, uint16_t *d_trace, void *stream,
                              char *err, size_t err_len);

/* julia_cuda_forward_device with every stage traced (the reference's --check traces the encoder
 * step by step and the head from the encoder's output, src/check.rs:177-224, :484-548, :564-596).
 * Any trace pointer may be NULL. d_trace: the residual stream after each encoder layer
 * [n_layers][n][D]; d_head_trace: the head's stream [n_head_layers + 1][nh][D], its input (final
 * LayerNorm + type embedding), then after each head layer, nh = the head's rows (n unless
 * julia_cuda_set_head_length limits them); d_scorer_trace: the scorer's hidden layer after GELU
 * for each marker [n_markers][scorer_hidden]. All f16. Slower: no CUDA graph. Returns 0 or -1. */
int julia_cuda_forward_trace(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                             const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                             int layer_fused, float *d_logits, uint16_t *d_trace,
                             uint16_t *d_head_trace, uint16_t *d_scorer_trace, void *stream,
                             char *err, size_t err_len);

/* One launch of a profiled forward (julia_cuda_forward_profile), in launch order. */
typedef struct jc_launch_info {
    uint32_t kind;   /* 0 GEMM, 1 attention, 2 embedding, 3 head input (final LayerNorm + type
                        embedding), 4 marker gather, 5 score, 6 trace copy */
    uint32_t epi;    /* GEMM: epilogue flags (JC_EPI_*) */
    uint32_t m, n, k; /* GEMM: rows, output columns, depth; attention: rows, heads, window;
                         edges: rows, width */
    int32_t layer;   /* encoder layer, -1 before the encoder, -2 the head and scorer */
    uint32_t ctas;   /* CTAs launched */
    uint32_t tile;   /* GEMM: tile rows << 16 | tile columns */
    uint32_t record; /* its first phase-stamp record (GEMM and attention launches, persistent
                        phases) */
    uint32_t launch;  /* the kernel launch it belongs to (a persistent launch logs one entry per
                         phase, all with its index) */
    uint32_t records; /* phase-stamp records it owns, from `record` on: a per-step launch's CTAs
                         (at most records_per_launch), a persistent phase's items */
    uint32_t items;   /* a persistent phase's work items (0 for per-step launches) */
} jc_launch_info;

/* A profiled forward (the reference's --time, src/timing.rs and src/profile.rs, with device-side
 * stamps as kernels/src/prof.rs). The forward's steps (julia_cuda_launches_per_forward of them in
 * per-step mode) own records_per_launch records of eight 64-bit words each in d_prof, step s the
 * records from s * records_per_launch on (d_prof: that many records for every step).
 *
 * julia_cuda_forward_profile runs the per-step kernels, captured into a CUDA graph with
 * programmatic dependent launch exactly as julia_cuda_run runs them; every GEMM and attention CTA
 * records [0] entry, [1] inputs ready (the previous kernel done), [2] first operand stage in shared
 * memory (GEMMs) / first tiles loaded (attention), [3] accumulator complete / key loop done, [4]
 * outputs written, [5] exit (%globaltimer ns, 0 where a stage does not apply), [6] the SM, [7] the
 * CTA's index (CTAs past records_per_launch are not recorded).
 *
 * julia_cuda_forward_profile_mode runs the forward in any mode (layer_fused 0, 1 or 2, as
 * julia_cuda_run_ex); the persistent kernel (not graphed here) records one record per work item,
 * in item order from its first step's records on (items past the launch's steps x
 * records_per_launch are not recorded): [0] item taken, [1] its inputs ready (dependency counters
 * reached), [2] first operand stage (GEMM tiles) / first tiles loaded (attention), [3] accumulator
 * complete / key loop done, [4] outputs written, [5] item reported, [6] the SM, [7] the CTA.
 *
 * info (info_cap entries) receives each launch's description, a persistent launch's one per
 * phase, and *n_launches their count. Waits for the forward. Returns 0 or -1. The stamps cost a
 * few global stores per CTA or item; a forward without a record array runs none. */
int julia_cuda_forward_profile(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                               const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                               float *d_logits, uint64_t *d_prof, uint32_t records_per_launch,
                               jc_launch_info *info, size_t info_cap, size_t *n_launches,
                               void *stream, char *err, size_t err_len);
int julia_cuda_forward_profile_mode(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                                    const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                                    int layer_fused, float *d_logits, uint64_t *d_prof,
                                    uint32_t records_per_launch, jc_launch_info *info,
                                    size_t info_cap, size_t *n_launches, void *stream, char *err,
                                    size_t err_len);

/* Failure detection: runs the persistent kernel with a grid barrier that waits for one CTA more
 * than the grid has, so every wait must give up after timeout_ns; writes the device error code it
 * recorded (JC_DEV_TIMEOUT_GRID = 4) and leaves the engine usable. No counterpart in the
 * reference (its grid barrier spins forever, kernels/src/gemm.rs:444-463). */
int julia_cuda_barrier_timeout_probe(JcEngine *engine, uint64_t timeout_ns, uint32_t *code,
                                     char *err, size_t err_len);

/* Waits for the engine's stream, then reads and clears the engine's own device error word into
 * *code (0: none; JC_DEV_* codes as jc_device_error). Every kernel an engine launches records
 * device-side timeouts in this word, not in the module's word that jc_device_error reads, so two
 * engines on one GPU (or an engine beside bare jc_* calls) each see only their own errors. On an
 * error it also re-zeroes the engine's persistent-kernel, split-K and split-KV counters.
 * julia_cuda_run checks the word itself after every queue of requests; callers of
 * julia_cuda_forward_device read it here. Returns 0, or -1. No counterpart in the reference. */
int julia_cuda_device_error(JcEngine *engine, uint32_t *code, char *err, size_t err_len);

/* Limits the head to the first `rows` rows of every later request (0: all rows, the default
 * and the reference's GPU behaviour, src/forward.rs:432-436): the final LayerNorm, the head
 * layers (their attention over those rows only) and the marker gather run on rows
 * [0, min(n, rows)), the encoder on all n. Markers must lie inside: julia_cuda_run rejects
 * others, and on the device path a marker outside records device error 6 (JC_DEV_BAD_INDEX,
 * read by jc_device_error; julia_cuda_run reports it) and is not read. Stands in for
 * julia-rs's head_length (passed to `sequence`, src/engine.rs:165), whose semantics are not in
 * the reference. Returns 0, or -1 for a NULL engine. */
int julia_cuda_set_head_length(JcEngine *engine, size_t rows);

/* Packs requests for throughput: julia_cuda_run then runs consecutive requests of one question
 * type as one forward of up to `rows` tokens (at most the engine's max_length; 0, the default,
 * runs each request alone as the reference does). Inside a packed forward every request attends
 * only to its own tokens and its RoPE positions start at 0, so each request's logits are its
 * own; gpu_ms reports the packed forward's time for each of its requests. Not combined with a
 * head length (requests then run alone). Returns 0, or -1 for a NULL engine or rows above
 * max_length. No counterpart in the reference (its engine runs requests one by one,
 * src/engine.rs:170-196). */
int julia_cuda_set_packing(JcEngine *engine, size_t rows);

/* How many kernels one forward pass launches (for launch accounting). */
int julia_cuda_launches_per_forward(const JcEngine *engine, uint32_t n, uint32_t n_markers,
                                    int layer_fused);
/* Model config and limits of an engine. */
int julia_cuda_engine_config(const JcEngine *engine, jc_model_config *cfg, size_t *max_length,
                             int *device, int *sms);

/* ============================ per-kernel entry points (device) ============================ */
/* Kernel-level boundary of the reference (src/gemm.rs:254 gemm::launch, kernels/src/main.rs:
 * 1043-1066 gemm_*(a, w, c, res, ws, counters, stats_in, colsum, stats_out, zero, zero_len, m, n,
 * k, eps, rope, bias)). Return 0, or -1 with jc_last_error(). */

/* Epilogue flags (kernels/src/main.rs:870-877). */
#define JC_EPI_RES 1u    /* c += a.w^T (res may alias c) */
#define JC_EPI_GEGLU 2u  /* c[:, j] = GELU(u_j) * g_j over interleaved Wi rows; c is [m, n/2] */
#define JC_EPI_LN 4u     /* LayerNorm folded: rstd * (acc - mean * colsum), stats from stats_in */
#define JC_EPI_STATS 8u  /* row sum / sum of squares of the stored f16 outputs added to stats_out */
#define JC_EPI_ROPE 16u  /* rotate-half RoPE on dims (i, i+32) of q and k heads (natural order) */
#define JC_EPI_BIAS 32u
#define JC_EPI_RELU 64u
#define JC_EPI_GELU 128u

/* c = epilogue(a . w^T): a [m, k] f16, w [n, k] f16, c [m, n] f16 ([m, n/2] for GEGLU), k a
 * multiple of 64. bn (32/64/128) and splits (1..8) of 0 choose automatically. ws / counters: the
 * split-K workspace (jc_gemm_ws_floats floats, jc_gemm_counters zeroed u32, kept zero between
 * calls; after jc_device_error reports a timeout the caller must zero the counters again: a split
 * that gave up never arrives, so its tile's counter stays non-zero). splits = -2 or -4 splits K across a thread-block cluster of that many CTAs instead, which
 * reduce their partials through distributed shared memory (64- or 128-column tiles; no workspace,
 * ws / counters unused; same result bits as that many workspace splits). stats_in / stats_out:
 * [m][2] f32 (sum, sum of squares). rope: 16 x m float4 (cos, sin of two pairs; jc_prep_rope_gemm).
 * zero / zero_len: a float buffer to clear on the way. Replaces src/gemm.rs:254-392. */
int jc_gemm(uint32_t epi, int bn, int splits, const uint16_t *a, const uint16_t *w, uint16_t *c,
            const uint16_t *res, float *ws, uint32_t *counters, const float *stats_in,
            const float *colsum, float *stats_out, float *zero, uint32_t zero_len, uint32_t m,
            uint32_t n, uint32_t k, float eps, const float *rope, const float *bias, void *stream);
/* jc_gemm for callers that cannot allocate device memory (a serving loop whose memory is planned
 * up front, or code where a cudaMalloc would synchronise or fail): the same arguments without
 * ws / counters. The split-K scratch is a fixed array in the library's own device memory (4 Mi
 * floats of partials + 4096 counters, 16 MiB per GPU, held until the process exits); a shape whose
 * split-K needs more is rejected with an error. Allocates nothing. The first call on a device
 * looks the array's address up (cudaGetSymbolAddress) and should come before any stream capture.
 * All calls share the array: calls that overlap on the GPU race. No counterpart in the reference. */
int jc_gemm_noalloc(uint32_t epi, int bn, int splits, const uint16_t *a, const uint16_t *w,
                    uint16_t *c, const uint16_t *res, const float *stats_in, const float *colsum,
                    float *stats_out, float *zero, uint32_t zero_len, uint32_t m, uint32_t n,
                    uint32_t k, float eps, const float *rope, const float *bias, void *stream);
/* One encoder layer on the persistent kernel, over device buffers the caller owns: the kernel-level
 * boundary of the reference's persistent `layer` kernel (kernels/src/main.rs:579-606, launched by
 * src/forward.rs:226-359; its plan, split-K and key-range arguments are this library's own
 * plan here). x [m][d_model] f16 is updated in place: qkv = RoPE(LN(x) Wqkv^T) (no LayerNorm when
 * qkv_colsum is NULL, as in layer 0), o = attention(qkv) (window 0: global, else keys within
 * +-window), x += o Wo^T, mbuf = GeGLU(LN(x) Wi^T), x += mbuf Wo_mlp^T. Scratch the caller owns:
 * qkv [m][3 d_model], o [m][d_model], mbuf [m][inter] f16. Statistics ([m][2] f32: sum and sum
 * of squares of the stored f16 rows): stats_mlp holds x's on entry (read when qkv_colsum is
 * given) and the updated x's on return; stats_attn is scratch (the statistics after the
 * attention block). Weights as prepared for the engine: wqkv [3 d_model][d_model] with the
 * LayerNorm's gamma folded (qkv_colsum [3 d_model]: f64 sums of its rounded rows), wo
 * [d_model][d_model], wi [2 inter][d_model] folded and interleaved for GeGLU
 * (jc_prep_interleave_geglu_f16; wi_colsum interleaved the same way), wo_mlp [d_model][inter].
 * rope: the GEMM layout of jc_gemm (16 x rope_stride float4, jc_prep_rope_gemm; rope_stride >= m,
 * 0 means m). d_model = 64 x heads; inter a multiple of 64. The phase descriptors, tensor maps
 * and completion counters live in a per-device scratch the library allocates on first use (and
 * grows with m): calls on one device must not overlap in time. Device-side timeouts (2 s) are
 * recorded in the module's error word (jc_device_error). Returns 0, or -1 (jc_last_error). */
int jc_layer(uint16_t *x, uint16_t *qkv, uint16_t *o, uint16_t *mbuf, float *stats_attn,
             float *stats_mlp, const uint16_t *wqkv, const float *qkv_colsum, const float *rope,
             uint32_t rope_stride, const uint16_t *wo, const uint16_t *wi, const float *wi_colsum,
             const uint16_t *wo_mlp, uint32_t m, uint32_t d_model, uint32_t heads, uint32_t inter,
             float eps, uint32_t window, void *stream);
size_t jc_gemm_ws_floats(uint32_t m, uint32_t n, uint32_t k, int bn, int splits);
size_t jc_gemm_counters(uint32_t m, uint32_t n, uint32_t k, int bn, int splits);
/* The persistent kernel's plan (the reference's LayerPlan / gemm_plan / phase_cost,
 * src/forward.rs:738-806, refit to the B200): the tile width (32 or 64 columns) a GEMM phase of m x
 * n x k with epilogue `epi` takes on a grid of `grid` CTAs, and the cost model behind it:
 * jc_gemm_phase_us, a launch's time in us (tiles in waves, a tile 0.8 us of first stage and drain,
 * 0.163 us per 64-deep k-block, 0.70 us of epilogue per 32 columns; the per-step kernels' model),
 * and jc_persist_phase_us, that plus 0.19 us for each item of a row block (what a persistent phase
 * pays for its items' reports). Both give -1 for a width they do not take or that does not divide
 * n. jc_persist_tile_policy sets the persistent kernel's width policy (0 the plan, 32 or 64 for
 * every phase that allows it) for later-planned launches and returns the previous one in place,
 * or -1 (and changes nothing) for any other value (a tuning and test hook; JC_PERSIST_BN sets the
 * starting policy). Host only. */
int jc_persist_tile(uint32_t m, uint32_t n, uint32_t k, uint32_t epi, uint32_t grid);
double jc_gemm_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid);
double jc_persist_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid);
void jc_persist_tile_policy(int *bn);
/* The tile height policy of later jc_gemm / jc_gemm_noalloc calls and later-captured engine
 * graphs: 0 automatic (64-row tiles for tiles of at most 64 columns without split-K whose 64-row
 * grid fits one wave, else 128), 128 (always 128 rows, the default) or 64 (64 rows wherever
 * legal). Sets *rows and returns the previous policy in place; other values are ignored. A tuning
 * and test hook (JC_GEMM_BM sets the starting policy). */
void jc_gemm_tile_rows(int *rows);
/* The CTA-pair policy of later jc_gemm / jc_gemm_noalloc calls and later-captured engine graphs:
 * 1 runs every unsplit 128- or 256-column launch on CTA pairs (tcgen05 cta_group::2: 256-row
 * tiles, each SM of a pair holding 128 rows and half of the weight tile), 0 (the default) the
 * launches that would otherwise run the single-SM persistent kernel with 256-column tiles (more
 * tiles than SMs: packs of thousands of rows), -1 none. Sets *policy and returns the previous one
 * in place; for any other value nothing changes and *policy becomes -2. A tuning and test hook
 * (JC_GEMM_PAIR sets the starting policy). No counterpart in the reference. */
void jc_gemm_pair_policy(int *policy);
/* The automatic choice (gemm::choose, src/gemm.rs:153-172, refit for the B200's SMs). */
int jc_choose_gemm(uint32_t m, uint32_t n, uint32_t k, int sms, int *bn, int *splits);

/* o = softmax(q k^T / 8) v per 64-wide head, qkv [n, 3*heads*64] (q | k | v, natural order),
 * o [n, heads*64]; window 0 = global, else keys with |q - k| <= window. kv_chunks > 1 splits the
 * keys into ranges (needs ws / counters, jc_attention_ws_floats / jc_attention_counters; counters
 * zero, kept zero, and to be zeroed again by the caller after jc_device_error reports a timeout);
 * 0 chooses. Replaces kernels/src/main.rs:303-542 and src/attn.rs:20-56. */
int jc_attention(const uint16_t *qkv, uint16_t *o, uint32_t n, uint32_t heads, uint32_t window,
                 uint32_t kv_chunks, float *ws, uint32_t *counters, void *stream);
size_t jc_attention_ws_floats(uint32_t n, uint32_t heads, uint32_t kv_chunks);
size_t jc_attention_counters(uint32_t n, uint32_t heads);
/* Which attention kernel serves a launch: the tcgen05 kernel (128-query tiles, S and P.V in
 * TMEM) for global attention from 832 tokens by default (JC_ATTN_TC_MIN), never for sliding
 * windows by default (JC_ATTN_TC_MIN_WINDOW); the mma.sync kernel otherwise. Sets the shortest
 * global and window sequence lengths for the tcgen05 kernel (1: every launch; 0xFFFFFFFF:
 * never) for later launches and later-captured engine graphs, and returns the previous ones in
 * place. A tuning and test hook. */
void jc_attention_tc_min(uint32_t *global_min, uint32_t *window_min);

/* x[i] = LayerNorm(table[ids[i]]) * gamma, f16; stats (optional) [n][2]. Replaces
 * kernels/src/main.rs:47-103 + src/lib.rs:164-219. */
int jc_embed(const uint32_t *ids, uint32_t n, const uint16_t *table, const float *gamma,
             uint32_t d, float eps, uint16_t *x, float *stats, void *stream);
/* out = LayerNorm(x) * gamma + add, stats [n][2] of out. Replaces kernels/src/main.rs:108-176. */
int jc_norm_add(const uint16_t *x, uint32_t n, uint32_t d, const float *gamma, const float *add,
                float eps, uint16_t *out, float *stats, void *stream);
/* logits[i] = y[markers[i]] . w + b. Replaces kernels/src/main.rs:180-200. */
int jc_score(const uint16_t *y, uint32_t d, const uint16_t *w, float b, const uint32_t *markers,
             uint32_t k, float *logits, void *stream);

/* The last error message of this thread. */
const char *jc_last_error(void);
/* Reads and clears the module's device error word on the current device (0: none): the word the
 * per-kernel entry points (jc_gemm, jc_attention, jc_gemm_noalloc, ...) record device-side
 * timeouts in. Engines keep their own (julia_cuda_device_error). */
int jc_device_error(uint32_t *code);

/* ============================== host weight preparation ============================== */
/* src/prep.rs. f16 outputs are bit patterns. */

/* W' = f16(w * gamma) ([out, k]), colsum[j] = sum_k W'[j, k] (f64 of the rounded values). */
void jc_prep_fold_layernorm(const float *w, const float *gamma, uint32_t out, uint32_t k,
                            uint16_t *w16, float *colsum);
/* Also bias' = b + W . beta (f64, from the f32 w). */
void jc_prep_fold_layernorm_bias(const float *w, const float *gamma, const float *beta,
                                 const float *b, uint32_t out, uint32_t k, uint16_t *w16,
                                 float *colsum, float *bias);
/* Wi rows [2I, k] (GELU inputs, then gates) in the GeGLU epilogue's order: packed row
 * 64t + 32s + e is source row 32t + e (+ I when s = 1). k = 1 reorders a vector. */
void jc_prep_interleave_geglu_f16(const uint16_t *w, uint32_t n, uint32_t k, uint16_t *out);
void jc_prep_interleave_geglu_f32(const float *w, uint32_t n, uint32_t k, float *out);
/* RoPE (cos, sin) table [n][32][2] in f32. */
void jc_prep_rope_table(float theta, uint32_t n, float *out);
/* The layout jc_gemm's rope argument takes, from a [>= m][32][2] table: float4 out[16][m] with
 * out[g][r] = (cos, sin) of pairs 2g and 2g + 1 of row r (pair-group major, so the rows a warp
 * handles are contiguous). The reference keeps its table row-major (src/prep.rs:88-118). */
void jc_prep_rope_gemm(const float *table, uint32_t m, float *out);

#ifdef __cplusplus
}
#endif
#endif /* JULIA_CUDA_H */
