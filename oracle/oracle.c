/*
 * CPU ORACLE for the julia-cuda encoder hot path. TEST INFRASTRUCTURE ONLY: loaded by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline legs; never by the product path.
 * What each function restates, with the reference file:line it follows, is in oracle.h.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* f16 */

uint16_t or_f16_from_f32(float x) {
    _Float16 h = (_Float16)x; /* IEEE round-to-nearest-even */
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

float or_f32_from_f16(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

void or_f16_round_array(const float *src, uint16_t *dst, size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) dst[i] = or_f16_from_f32(src[i]);
}

static float *f16_to_f32_alloc(const uint16_t *src, size_t n) {
    float *d = (float *)malloc(n * sizeof(float));
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) d[i] = or_f32_from_f16(src[i]);
    return d;
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------------------------ */
/* layout and random init */

int or_layout_of(const or_config *c, or_layout *o) {
    if (c->n_layers > OR_MAX_LAYERS || c->n_head_layers > OR_MAX_HEAD || c->d_model % 64 ||
        c->n_heads * 64 != c->d_model)
        return -1;
    memset(o, 0, sizeof(*o));
    size_t at = 0;
    const size_t D = (size_t)c->d_model, I = (size_t)c->inter, F = (size_t)c->head_ff,
                 S = (size_t)c->scorer_hidden;
#define PUT(span, n) do { (span).off = at; (span).len = (n); at += (n); } while (0)
    PUT(o->tok_emb, (size_t)c->vocab * D);
    PUT(o->emb_norm, D);
    for (int l = 0; l < c->n_layers; l++) {
        PUT(o->attn_norm[l], l == 0 ? 0 : D); /* ModernBERT's first layer has no attention norm */
        PUT(o->wqkv[l], 3 * D * D);
        PUT(o->wo[l], D * D);
        PUT(o->mlp_norm[l], D);
        PUT(o->wi[l], 2 * I * D);
        PUT(o->wo_mlp[l], D * I);
    }
    PUT(o->final_norm, D);
    PUT(o->type_emb, (size_t)c->n_qtypes * D);
    for (int l = 0; l < c->n_head_layers; l++) {
        PUT(o->h_norm1_w[l], D);
        PUT(o->h_norm1_b[l], D);
        PUT(o->h_in_w[l], 3 * D * D);
        PUT(o->h_in_b[l], 3 * D);
        PUT(o->h_out_w[l], D * D);
        PUT(o->h_out_b[l], D);
        PUT(o->h_norm2_w[l], D);
        PUT(o->h_norm2_b[l], D);
        PUT(o->h_l1_w[l], F * D);
        PUT(o->h_l1_b[l], F);
        PUT(o->h_l2_w[l], D * F);
        PUT(o->h_l2_b[l], D);
    }
    PUT(o->s_norm_w, D);
    PUT(o->s_norm_b, D);
    PUT(o->s_lin1_w, S * D);
    PUT(o->s_lin1_b, S);
    PUT(o->s_lin2_w, S);
    PUT(o->s_lin2_b, 1);
#undef PUT
    o->total = at;
    return 0;
}

size_t or_raw_size(const or_config *c) {
    or_layout o;
    if (or_layout_of(c, &o)) return 0;
    return o.total;
}

static inline uint64_t fmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

/* Counter-based normal: element i of stream `seed`, Box-Muller on two hashed uniforms. */
static inline float normal_at(uint64_t seed, size_t i) {
    uint64_t r1 = fmix64(seed + 0x9e3779b97f4a7c15ULL * (2 * (uint64_t)i + 1));
    uint64_t r2 = fmix64(seed + 0x9e3779b97f4a7c15ULL * (2 * (uint64_t)i + 2));
    double u1 = ((double)(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0, 1] */
    double u2 = (double)(r2 >> 11) * (1.0 / 9007199254740992.0);
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

void or_fill_normal(float *dst, size_t n, uint64_t seed, float mean, float std) {
    uint64_t s = fmix64(seed ^ 0x5bd1e9955bd1e995ULL);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) dst[i] = mean + std * normal_at(s, i);
}

static void fill_span(float *raw, or_span sp, uint64_t seed, int tensor, float mean, float std) {
    if (!sp.len) return;
    or_fill_normal(raw + sp.off, sp.len, seed * 0x100000001b3ULL + (uint64_t)tensor * 7919, mean,
                   std);
}

void or_init_random(const or_config *c, uint64_t seed, float *raw) {
    or_layout o;
    if (or_layout_of(c, &o)) return;
    int t = 0;
    const float W = 0.02f, G = 0.05f;
    fill_span(raw, o.tok_emb, seed, t++, 0.f, W);
    fill_span(raw, o.emb_norm, seed, t++, 1.f, G);
    for (int l = 0; l < c->n_layers; l++) {
        fill_span(raw, o.attn_norm[l], seed, t++, 1.f, G);
        fill_span(raw, o.wqkv[l], seed, t++, 0.f, W);
        fill_span(raw, o.wo[l], seed, t++, 0.f, W);
        fill_span(raw, o.mlp_norm[l], seed, t++, 1.f, G);
        fill_span(raw, o.wi[l], seed, t++, 0.f, W);
        fill_span(raw, o.wo_mlp[l], seed, t++, 0.f, W);
    }
    fill_span(raw, o.final_norm, seed, t++, 1.f, G);
    fill_span(raw, o.type_emb, seed, t++, 0.f, W);
    for (int l = 0; l < c->n_head_layers; l++) {
        fill_span(raw, o.h_norm1_w[l], seed, t++, 1.f, G);
        fill_span(raw, o.h_norm1_b[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_in_w[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_in_b[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_out_w[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_out_b[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_norm2_w[l], seed, t++, 1.f, G);
        fill_span(raw, o.h_norm2_b[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_l1_w[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_l1_b[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_l2_w[l], seed, t++, 0.f, W);
        fill_span(raw, o.h_l2_b[l], seed, t++, 0.f, W);
    }
    fill_span(raw, o.s_norm_w, seed, t++, 1.f, G);
    fill_span(raw, o.s_norm_b, seed, t++, 0.f, W);
    fill_span(raw, o.s_lin1_w, seed, t++, 0.f, W);
    fill_span(raw, o.s_lin1_b, seed, t++, 0.f, W);
    fill_span(raw, o.s_lin2_w, seed, t++, 0.f, W);
    fill_span(raw, o.s_lin2_b, seed, t++, 0.f, W);
}

/* ------------------------------------------------------------------------------------------ */
/* math pieces */

/* Abramowitz & Stegun 7.1.26 erf, GELU(x) = x * Phi(x); the kernels' formula (the reference's
 * kernels/src/gemm.rs:139-150, host f64 version src/check.rs:931-945). */
float or_gelu(float xf) {
    double x = xf;
    double t = 1.0 / (1.0 + 0.2316419 * fabs(x));
    double p = (((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t +
               0.254829592;
    p *= t;
    double q = 0.5 * p * exp(-x * x / 2.0);
    return (float)(x * (x >= 0 ? 1.0 - q : q));
}

void or_rope_table(float theta, int n, float *out) {
    float inv[32];
    for (int j = 0; j < 32; j++) inv[j] = 1.0f / powf(theta, (float)(2 * j) / 64.0f);
    for (int p = 0; p < n; p++)
        for (int j = 0; j < 32; j++) {
            float a = (float)p * inv[j];
            out[(p * 32 + j) * 2] = cosf(a);
            out[(p * 32 + j) * 2 + 1] = sinf(a);
        }
}

/* y[m,n] (+)= x[m,k] . w[n,k]^T (+ bias), f32, 4x4 register blocks, vectorized along k. */
typedef float v8f __attribute__((vector_size(32)));

static inline float hsum8(v8f v) {
    return ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
}

static void matmul_f32(const float *x, int m, int k, const float *w, int n, float *y,
                       const float *bias, int accumulate) {
    const int kv = k / 8 * 8;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int jb = 0; jb < (n + 3) / 4; jb++) {
        for (int ib = 0; ib < (m + 3) / 4; ib++) {
            int i0 = ib * 4, j0 = jb * 4;
            int ni = m - i0 < 4 ? m - i0 : 4, nj = n - j0 < 4 ? n - j0 : 4;
            v8f acc[4][4];
            memset(acc, 0, sizeof(acc));
            for (int p = 0; p < kv; p += 8) {
                v8f xv[4], wv[4];
                for (int a = 0; a < 4; a++) {
                    int ii = i0 + (a < ni ? a : 0), jj = j0 + (a < nj ? a : 0);
                    memcpy(&xv[a], x + (size_t)ii * k + p, 32);
                    memcpy(&wv[a], w + (size_t)jj * k + p, 32);
                }
                for (int a = 0; a < 4; a++)
                    for (int b = 0; b < 4; b++) acc[a][b] += xv[a] * wv[b];
            }
            for (int a = 0; a < ni; a++)
                for (int b = 0; b < nj; b++) {
                    float s = hsum8(acc[a][b]);
                    const float *xr = x + (size_t)(i0 + a) * k, *wr = w + (size_t)(j0 + b) * k;
                    for (int p = kv; p < k; p++) s += xr[p] * wr[p];
                    if (bias) s += bias[j0 + b];
                    float *dst = y + (size_t)(i0 + a) * n + j0 + b;
                    *dst = accumulate ? *dst + s : s;
                }
        }
    }
}

/* LayerNorm rows in f64 (src/check.rs:227-242): out = (x - mean) * r * gamma (+ beta). */
static void layernorm_rows(const float *x, int n, int d, const float *gamma, const float *beta,
                           float eps, float *out) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        const float *r = x + (size_t)i * d;
        double mean = 0, var = 0;
        for (int j = 0; j < d; j++) mean += r[j];
        mean /= d;
        for (int j = 0; j < d; j++) var += (r[j] - mean) * (r[j] - mean);
        var /= d;
        double rs = 1.0 / sqrt(var + (double)eps);
        for (int j = 0; j < d; j++)
            out[(size_t)i * d + j] =
                (float)((r[j] - mean) * rs * gamma[j] + (beta ? (double)beta[j] : 0.0));
    }
}

/* Rotate-half RoPE on dims (i, i + 32) of every head of the q and k thirds of a [n, 3D] row. */
static void rope_apply_f32(float *qkv, int n, int D, const float *table) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; r++) {
        float *row = qkv + (size_t)r * 3 * D;
        for (int h = 0; h < 2 * D / 64; h++)
            for (int i = 0; i < 32; i++) {
                float cs = table[(r * 32 + i) * 2], sn = table[(r * 32 + i) * 2 + 1];
                float x1 = row[h * 64 + i], x2 = row[h * 64 + i + 32];
                row[h * 64 + i] = x1 * cs - x2 * sn;
                row[h * 64 + i + 32] = x2 * cs + x1 * sn;
            }
    }
}

static inline int key_allowed(int q, int key, int window) {
    if (window <= 0) return 1;
    int d = q > key ? q - key : key - q;
    return d <= window;
}

void or_attention_f32(const float *qkv, float *o, int n, int heads, int window) {
    const int D = heads * 64;
#pragma omp parallel
    {
        float *s = (float *)malloc((size_t)n * sizeof(float));
#pragma omp for collapse(2) schedule(dynamic, 4)
        for (int h = 0; h < heads; h++)
            for (int i = 0; i < n; i++) {
                const float *q = qkv + (size_t)i * 3 * D + h * 64;
                float mx = -INFINITY;
                for (int j = 0; j < n; j++) {
                    if (!key_allowed(i, j, window)) { s[j] = -INFINITY; continue; }
                    const float *kk = qkv + (size_t)j * 3 * D + D + h * 64;
                    float acc = 0;
                    for (int e = 0; e < 64; e++) acc += q[e] * kk[e];
                    s[j] = acc / 8.0f;
                    if (s[j] > mx) mx = s[j];
                }
                float sum = 0, out[64] = {0};
                for (int j = 0; j < n; j++) {
                    if (s[j] == -INFINITY) continue;
                    float p = expf(s[j] - mx);
                    sum += p;
                    const float *v = qkv + (size_t)j * 3 * D + 2 * D + h * 64;
                    for (int e = 0; e < 64; e++) out[e] += p * v[e];
                }
                for (int e = 0; e < 64; e++) o[(size_t)i * D + h * 64 + e] = out[e] / sum;
            }
        free(s);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* f32 model */

int or_forward_f32_full(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, float *head_trace, float *scorer_trace) {
    or_layout L;
    if (or_layout_of(c, &L) || n <= 0 || n > c->max_positions || qtype < 0 ||
        qtype >= c->n_qtypes)
        return -1;
    for (int i = 0; i < n; i++)
        if (ids[i] >= (uint32_t)c->vocab) return -1;
    /* the head runs on rows [0, nh) (all rows unless head_rows limits it) */
    const int nh = head_rows > 0 && head_rows < n ? head_rows : n;
    for (int i = 0; i < n_markers; i++)
        if (markers[i] >= (uint32_t)nh) return -1;
    const int D = c->d_model, I = c->inter, F = c->head_ff, S = c->scorer_hidden;
    const int H = c->n_heads;
    float *x = malloc((size_t)n * D * 4), *h = malloc((size_t)n * D * 4);
    float *qkv = malloc((size_t)n * 3 * D * 4), *o = malloc((size_t)n * D * 4);
    size_t big = (size_t)n * (2 * I > F ? 2 * I : F);
    float *hh = malloc(big * 4), *mm = malloc((size_t)n * I * 4);
    float *rg = malloc((size_t)n * 64 * 4), *rl = malloc((size_t)n * 64 * 4);
    or_rope_table(c->theta_global, n, rg);
    or_rope_table(c->theta_local, n, rl);

    /* embed: LN(table[id]) * gamma (no bias) */
    for (int i = 0; i < n; i++) memcpy(h + (size_t)i * D, raw + L.tok_emb.off + (size_t)ids[i] * D, D * 4);
    layernorm_rows(h, n, D, raw + L.emb_norm.off, NULL, c->norm_eps, x);

    for (int l = 0; l < c->n_layers; l++) {
        int global = l % c->global_every == 0;
        if (L.attn_norm[l].len)
            layernorm_rows(x, n, D, raw + L.attn_norm[l].off, NULL, c->norm_eps, h);
        else
            memcpy(h, x, (size_t)n * D * 4);
        matmul_f32(h, n, D, raw + L.wqkv[l].off, 3 * D, qkv, NULL, 0);
        rope_apply_f32(qkv, n, D, global ? rg : rl);
        or_attention_f32(qkv, o, n, H, global ? 0 : c->window);
        matmul_f32(o, n, D, raw + L.wo[l].off, D, x, NULL, 1);
        layernorm_rows(x, n, D, raw + L.mlp_norm[l].off, NULL, c->norm_eps, h);
        matmul_f32(h, n, D, raw + L.wi[l].off, 2 * I, hh, NULL, 0);
#pragma omp parallel for schedule(static)
        for (int r = 0; r < n; r++)
            for (int j = 0; j < I; j++)
                mm[(size_t)r * I + j] =
                    or_gelu(hh[(size_t)r * 2 * I + j]) * hh[(size_t)r * 2 * I + I + j];
        matmul_f32(mm, n, I, raw + L.wo_mlp[l].off, D, x, NULL, 1);
        if (trace_x) memcpy(trace_x + (size_t)l * n * D, x, (size_t)n * D * 4);
    }

    /* head input: final LN (encoder eps) + type embedding */
    layernorm_rows(x, nh, D, raw + L.final_norm.off, NULL, c->norm_eps, h);
    const float *te = raw + L.type_emb.off + (size_t)qtype * D;
    for (int i = 0; i < nh; i++)
        for (int j = 0; j < D; j++) x[(size_t)i * D + j] = h[(size_t)i * D + j] + te[j];
    if (head_trace) memcpy(head_trace, x, (size_t)nh * D * 4);
    for (int l = 0; l < c->n_head_layers; l++) {
        layernorm_rows(x, nh, D, raw + L.h_norm1_w[l].off, raw + L.h_norm1_b[l].off, c->head_eps, h);
        matmul_f32(h, nh, D, raw + L.h_in_w[l].off, 3 * D, qkv, raw + L.h_in_b[l].off, 0);
        or_attention_f32(qkv, o, nh, H, 0);
        matmul_f32(o, nh, D, raw + L.h_out_w[l].off, D, x, raw + L.h_out_b[l].off, 1);
        layernorm_rows(x, nh, D, raw + L.h_norm2_w[l].off, raw + L.h_norm2_b[l].off, c->head_eps, h);
        matmul_f32(h, nh, D, raw + L.h_l1_w[l].off, F, hh, raw + L.h_l1_b[l].off, 0);
        for (size_t i = 0; i < (size_t)nh * F; i++) hh[i] = hh[i] > 0 ? hh[i] : 0;
        matmul_f32(hh, nh, F, raw + L.h_l2_w[l].off, D, x, raw + L.h_l2_b[l].off, 1);
        if (head_trace) memcpy(head_trace + (size_t)(l + 1) * nh * D, x, (size_t)nh * D * 4);
    }
    /* scorer on the marker rows */
    float *z = malloc((size_t)(n_markers ? n_markers : 1) * D * 4);
    float *zn = malloc((size_t)(n_markers ? n_markers : 1) * D * 4);
    float *y = malloc((size_t)(n_markers ? n_markers : 1) * S * 4);
    for (int i = 0; i < n_markers; i++) memcpy(z + (size_t)i * D, x + (size_t)markers[i] * D, D * 4);
    layernorm_rows(z, n_markers, D, raw + L.s_norm_w.off, raw + L.s_norm_b.off, c->head_eps, zn);
    matmul_f32(zn, n_markers, D, raw + L.s_lin1_w.off, S, y, raw + L.s_lin1_b.off, 0);
    for (size_t i = 0; i < (size_t)n_markers * S; i++) y[i] = or_gelu(y[i]);
    if (scorer_trace) memcpy(scorer_trace, y, (size_t)n_markers * S * 4);
    matmul_f32(y, n_markers, S, raw + L.s_lin2_w.off, 1, logits, raw + L.s_lin2_b.off, 0);
    free(z); free(zn); free(y);
    free(x); free(h); free(qkv); free(o); free(hh); free(mm); free(rg); free(rl);
    return 0;
}

int or_forward_f32_head(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x) {
    return or_forward_f32_full(c, raw, ids, n, markers, n_markers, qtype, head_rows, logits,
                               trace_x, NULL, NULL);
}

int or_forward_f32(const or_config *c, const float *raw, const uint32_t *ids, int n,
                   const uint32_t *markers, int n_markers, int qtype, float *logits,
                   float *trace_x) {
    return or_forward_f32_head(c, raw, ids, n, markers, n_markers, qtype, 0, logits, trace_x);
}

/* ------------------------------------------------------------------------------------------ */
/* f16 emulation of the kernels' arithmetic */

void or_row_stats(const uint16_t *x, int n, int d, float *stats) {
    for (int i = 0; i < n; i++) {
        float s = 0, q = 0;
        for (int j = 0; j < d; j++) {
            float v = or_f32_from_f16(x[(size_t)i * d + j]);
            s += v;
            q = fmaf(v, v, q);
        }
        stats[2 * i] = s;
        stats[2 * i + 1] = q;
    }
}

/* acc[m][n] = sum_p a[i,p] * w[j,p]: exact f16 products, summed in f64, rounded to f32. */
static void gemm_acc_f16(const uint16_t *a16, const uint16_t *w16, int m, int n, int k,
                         float *acc) {
    float *a = f16_to_f32_alloc(a16, (size_t)m * k), *w = f16_to_f32_alloc(w16, (size_t)n * k);
    typedef double v4d __attribute__((vector_size(32)));
    typedef float v4f __attribute__((vector_size(16)));
    const int kv = k / 4 * 4;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int jb = 0; jb < (n + 3) / 4; jb++)
        for (int ib = 0; ib < (m + 3) / 4; ib++) {
            int i0 = ib * 4, j0 = jb * 4;
            int ni = m - i0 < 4 ? m - i0 : 4, nj = n - j0 < 4 ? n - j0 : 4;
            v4d s[4][4];
            memset(s, 0, sizeof(s));
            for (int p = 0; p < kv; p += 4) {
                v4f av[4], wv[4];
                for (int q = 0; q < 4; q++) {
                    int ii = i0 + (q < ni ? q : 0), jj = j0 + (q < nj ? q : 0);
                    memcpy(&av[q], a + (size_t)ii * k + p, 16);
                    memcpy(&wv[q], w + (size_t)jj * k + p, 16);
                }
                for (int x = 0; x < 4; x++)
                    for (int y = 0; y < 4; y++)
                        s[x][y] += __builtin_convertvector(av[x] * wv[y], v4d);
            }
            for (int x = 0; x < ni; x++)
                for (int y = 0; y < nj; y++) {
                    double t = (s[x][y][0] + s[x][y][1]) + (s[x][y][2] + s[x][y][3]);
                    for (int p = kv; p < k; p++)
                        t += (double)(a[(size_t)(i0 + x) * k + p] * w[(size_t)(j0 + y) * k + p]);
                    acc[(size_t)(i0 + x) * n + j0 + y] = (float)t;
                }
        }
    free(a);
    free(w);
}

void or_emu_gemm(int epi, const uint16_t *a, const uint16_t *w, uint16_t *c, int m, int n, int k,
                 const float *stats_in, const float *colsum, float eps, const float *rope,
                 const float *bias, float *stats_out) {
    float *acc = malloc((size_t)m * n * 4);
    gemm_acc_f16(a, w, m, n, k, acc);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < m; r++) {
        float *v = acc + (size_t)r * n;
        if (epi & OR_LN) {
            float mean = stats_in[2 * r] / k;
            float var = stats_in[2 * r + 1] / k - mean * mean;
            float rstd = 1.0f / sqrtf((var > 0 ? var : 0) + eps);
            for (int j = 0; j < n; j++) v[j] = rstd * (v[j] - mean * colsum[j]);
        }
        if (epi & OR_BIAS)
            for (int j = 0; j < n; j++) v[j] += bias[j];
        if (epi & OR_RELU)
            for (int j = 0; j < n; j++) v[j] = v[j] > 0 ? v[j] : 0;
        if (epi & OR_GELU)
            for (int j = 0; j < n; j++) v[j] = or_gelu(v[j]);
        if (epi & OR_ROPE) {
            for (int h = 0; h < 2 * (n / 3) / 64; h++)
                for (int i = 0; i < 32; i++) {
                    float cs = rope[(r * 32 + i) * 2], sn = rope[(r * 32 + i) * 2 + 1];
                    float x1 = v[h * 64 + i], x2 = v[h * 64 + i + 32];
                    v[h * 64 + i] = x1 * cs - x2 * sn;
                    v[h * 64 + i + 32] = x2 * cs + x1 * sn;
                }
        }
        if (epi & OR_GEGLU) {
            int half = n / 2;
            for (int j = 0; j < half; j++)
                c[(size_t)r * half + j] = or_f16_from_f32(or_gelu(v[j]) * v[half + j]);
        } else {
            float s = 0, q = 0;
            for (int j = 0; j < n; j++) {
                float o = v[j];
                if (epi & OR_RES) o += or_f32_from_f16(c[(size_t)r * n + j]);
                uint16_t b = or_f16_from_f32(o);
                c[(size_t)r * n + j] = b;
                float st = or_f32_from_f16(b);
                s += st;
                q = fmaf(st, st, q);
            }
            if (epi & OR_STATS) {
                stats_out[2 * r] += s;
                stats_out[2 * r + 1] += q;
            }
        }
    }
    free(acc);
}

void or_emu_attention(const uint16_t *qkv, uint16_t *o, int n, int heads, int window) {
    const int D = heads * 64;
#pragma omp parallel
    {
        float *s = (float *)malloc((size_t)n * sizeof(float));
#pragma omp for collapse(2) schedule(dynamic, 4)
        for (int h = 0; h < heads; h++)
            for (int i = 0; i < n; i++) {
                float q[64];
                for (int e = 0; e < 64; e++) q[e] = or_f32_from_f16(qkv[(size_t)i * 3 * D + h * 64 + e]);
                float mx = -INFINITY;
                for (int j = 0; j < n; j++) {
                    if (!key_allowed(i, j, window)) { s[j] = -INFINITY; continue; }
                    const uint16_t *kk = qkv + (size_t)j * 3 * D + D + h * 64;
                    float acc = 0;
                    for (int e = 0; e < 64; e++) acc += q[e] * or_f32_from_f16(kk[e]);
                    s[j] = acc / 8.0f;
                    if (s[j] > mx) mx = s[j];
                }
                float sum = 0, out[64] = {0};
                for (int j = 0; j < n; j++) {
                    if (s[j] == -INFINITY) continue;
                    float p = expf(s[j] - mx);
                    sum += p;
                    float p16 = or_f32_from_f16(or_f16_from_f32(p));
                    const uint16_t *v = qkv + (size_t)j * 3 * D + 2 * D + h * 64;
                    for (int e = 0; e < 64; e++) out[e] += p16 * or_f32_from_f16(v[e]);
                }
                for (int e = 0; e < 64; e++)
                    o[(size_t)i * D + h * 64 + e] = or_f16_from_f32(out[e] / sum);
            }
        free(s);
    }
}

void or_emu_embed(const uint16_t *table, const float *gamma, const uint32_t *ids, int n, int d,
                  float eps, uint16_t *x) {
    for (int i = 0; i < n; i++) {
        const uint16_t *r = table + (size_t)ids[i] * d;
        float mean = 0, var = 0;
        for (int j = 0; j < d; j++) mean += or_f32_from_f16(r[j]);
        mean /= d;
        for (int j = 0; j < d; j++) {
            float t = or_f32_from_f16(r[j]) - mean;
            var += t * t;
        }
        var /= d;
        float rstd = 1.0f / sqrtf(var + eps);
        for (int j = 0; j < d; j++)
            x[(size_t)i * d + j] = or_f16_from_f32((or_f32_from_f16(r[j]) - mean) * rstd * gamma[j]);
    }
}

void or_emu_norm_add(const uint16_t *x, const float *gamma, const float *add, int n, int d,
                     float eps, uint16_t *out, float *stats) {
    for (int i = 0; i < n; i++) {
        const uint16_t *r = x + (size_t)i * d;
        float mean = 0, var = 0;
        for (int j = 0; j < d; j++) mean += or_f32_from_f16(r[j]);
        mean /= d;
        for (int j = 0; j < d; j++) {
            float t = or_f32_from_f16(r[j]) - mean;
            var += t * t;
        }
        var /= d;
        float rstd = 1.0f / sqrtf(var + eps), s = 0, q = 0;
        for (int j = 0; j < d; j++) {
            uint16_t b = or_f16_from_f32((or_f32_from_f16(r[j]) - mean) * rstd * gamma[j] + add[j]);
            out[(size_t)i * d + j] = b;
            float v = or_f32_from_f16(b);
            s += v;
            q = fmaf(v, v, q);
        }
        stats[2 * i] = s;
        stats[2 * i + 1] = q;
    }
}

void or_emu_score(const uint16_t *y, const uint16_t *w, float b, const uint32_t *markers, int k,
                  int d, float *logits) {
    for (int i = 0; i < k; i++) {
        float acc = 0;
        for (int j = 0; j < d; j++)
            acc += or_f32_from_f16(y[(size_t)markers[i] * d + j]) * or_f32_from_f16(w[j]);
        logits[i] = acc + b;
    }
}

/* ------------------------------------------------------------------------------------------ */
/* weight preparation (src/prep.rs) */

void or_fold_layernorm(const float *w, const float *gamma, int out, int k, uint16_t *w16,
                       float *colsum) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < out; j++) {
        double s = 0;
        for (int p = 0; p < k; p++) {
            uint16_t b = or_f16_from_f32(w[(size_t)j * k + p] * gamma[p]);
            w16[(size_t)j * k + p] = b;
            s += (double)or_f32_from_f16(b);
        }
        colsum[j] = (float)s;
    }
}

void or_fold_layernorm_bias(const float *w, const float *gamma, const float *beta, const float *b,
                            int out, int k, uint16_t *w16, float *colsum, float *bias) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < out; j++) {
        double wb = 0;
        for (int p = 0; p < k; p++) wb += (double)w[(size_t)j * k + p] * (double)beta[p];
        bias[j] = (float)((double)b[j] + wb);
    }
    or_fold_layernorm(w, gamma, out, k, w16, colsum);
}

/* src/prep.rs:88-101: packed row p of a q or k head holds dim p/2 + (p%2)*32. */
void or_ref_permute_rope_rows(int n, int32_t *src) {
    for (int p = 0; p < n; p++) {
        if (p < 2 * n / 3) {
            int head = p / 64, i = p % 64;
            src[p] = head * 64 + i / 2 + (i % 2) * 32;
        } else {
            src[p] = p;
        }
    }
}

/* src/prep.rs:67-77: packed row p = 64t + 32h + 16q + 8s + e is source row 32t + 16h + 8q + e
 * (+ inter for the gate, s = 1). */
void or_ref_interleave_geglu_rows(int n, int32_t *src) {
    int inter = n / 2;
    for (int p = 0; p < n; p++) {
        int t = p / 64, h = (p % 64) / 32, q = (p % 32) / 16, s = (p % 16) / 8, e = p % 8;
        src[p] = t * 32 + h * 16 + q * 8 + e + (s ? inter : 0);
    }
}

/* src/forward.rs:783-806 */
double or_ref_phase_cost(int n, int cols, int k, int bm, int z, int sms, int per_sm) {
    long tasks = (long)(cols / 64) * ((n + bm - 1) / bm) * z;
    double steps = (double)(k / 32) / z;
    double task = (bm == 32 ? 5.0 : 10.0) + 0.35 * steps;
    long on_sm = (tasks + sms - 1) / sms;
    long rounds = on_sm / per_sm, rest = on_sm % per_sm;
    double t = rounds * (1.0 + 0.2 * (per_sm - 1)) * task;
    if (rest > 0) t += (1.0 + 0.2 * (rest - 1)) * task;
    if (z > 1) t += 0.4 * z * (bm / 32);
    return t;
}

/* src/forward.rs:761-769: min cost over bm in {32, 64}, z in 1..=4 with >= 3 K steps per split;
 * the first minimum in that order wins. */
void or_ref_gemm_plan(int n, int cols, int k, int sms, int per_sm, int *bm_out, int *z_out) {
    double best = INFINITY;
    int bb = 32, bz = 1;
    const int bms[2] = {32, 64};
    for (int a = 0; a < 2; a++)
        for (int z = 1; z <= 4; z++) {
            if (k / 32 / z < 3) continue;
            double c = or_ref_phase_cost(n, cols, k, bms[a], z, sms, per_sm);
            if (c < best) { best = c; bb = bms[a]; bz = z; }
        }
    *bm_out = bb;
    *z_out = bz;
}

/* ------------------------------------------------------------------------------------------ */
/* the whole f16-emulated forward pass */

int or_forward_emu_full(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, float *head_trace, float *scorer_trace,
                        int bugs) {
    or_layout L;
    if (or_layout_of(c, &L) || n <= 0 || n > c->max_positions || qtype < 0 ||
        qtype >= c->n_qtypes)
        return -1;
    for (int i = 0; i < n; i++)
        if (ids[i] >= (uint32_t)c->vocab) return -1;
    const int nh = head_rows > 0 && head_rows < n ? head_rows : n;
    for (int i = 0; i < n_markers; i++)
        if (markers[i] >= (uint32_t)nh) return -1;
    const int D = c->d_model, I = c->inter, F = c->head_ff, S = c->scorer_hidden, H = c->n_heads;
    const size_t nD = (size_t)n * D;
    uint16_t *x = malloc(nD * 2), *qkv = malloc(nD * 3 * 2), *o = malloc(nD * 2);
    uint16_t *m = malloc((size_t)n * (I > F ? I : F) * 2), *y = malloc((size_t)n * S * 2);
    float *st_a = calloc((size_t)2 * n, 4), *st_b = calloc((size_t)2 * n, 4);
    float *rg = malloc((size_t)n * 64 * 4), *rl = malloc((size_t)n * 64 * 4);
    or_rope_table(c->theta_global, n, rg);
    or_rope_table(c->theta_local, n, rl);
    size_t wmax = (size_t)(2 * I > F ? 2 * I : F) * D;
    if ((size_t)3 * D * D > wmax) wmax = (size_t)3 * D * D;
    if ((size_t)D * F > wmax) wmax = (size_t)D * F;
    uint16_t *w16 = malloc(wmax * 2);
    float *colsum = malloc((size_t)(3 * D > 2 * I ? 3 * D : 2 * I) * 4 + (size_t)F * 4 + (size_t)S * 4);
    float *bias = malloc((size_t)(3 * D > F ? 3 * D : F) * 4 + (size_t)S * 4 + 64);
    float *wtmp = malloc(wmax * 4);

    /* embed */
    uint16_t *table = malloc((size_t)c->vocab * D * 2);
    or_f16_round_array(raw + L.tok_emb.off, table, (size_t)c->vocab * D);
    or_emu_embed(table, raw + L.emb_norm.off, ids, n, D, c->norm_eps, x);
    free(table);
    /* st_b plays the reference's stats_mlp (feeds qkv), st_a stats_attn (feeds wi). */
    or_row_stats(x, n, D, st_b);

    for (int l = 0; l < c->n_layers; l++) {
        int global = l % c->global_every == 0;
        const float *rope = global ? rg : rl;
        int epi = OR_ROPE;
        if (bugs & 2) epi = 0;
        if (L.attn_norm[l].len) {
            or_fold_layernorm(raw + L.wqkv[l].off, raw + L.attn_norm[l].off, 3 * D, D, w16, colsum);
            epi |= OR_LN;
        } else {
            or_f16_round_array(raw + L.wqkv[l].off, w16, (size_t)3 * D * D);
        }
        or_emu_gemm(epi, x, w16, qkv, n, 3 * D, D, st_b, colsum, c->norm_eps, rope, NULL, NULL);
        or_emu_attention(qkv, o, n, H, (global || (bugs & 4)) ? 0 : c->window);
        or_f16_round_array(raw + L.wo[l].off, w16, (size_t)D * D);
        memset(st_a, 0, (size_t)2 * n * 4);
        or_emu_gemm(OR_RES | OR_STATS, o, w16, x, n, D, D, NULL, NULL, 0, NULL, NULL, st_a);
        or_fold_layernorm(raw + L.wi[l].off, raw + L.mlp_norm[l].off, 2 * I, D, w16, colsum);
        if (bugs & 1) { /* the wrong GeGLU half as the GELU input */
            memcpy(wtmp, w16, (size_t)I * D * 2);
            memmove(w16, w16 + (size_t)I * D, (size_t)I * D * 2);
            memcpy(w16 + (size_t)I * D, wtmp, (size_t)I * D * 2);
            float *ct = bias;
            memcpy(ct, colsum, (size_t)I * 4);
            memmove(colsum, colsum + I, (size_t)I * 4);
            memcpy(colsum + I, ct, (size_t)I * 4);
        }
        or_emu_gemm(OR_LN | OR_GEGLU, x, w16, m, n, 2 * I, D, st_a, colsum, c->norm_eps, NULL,
                    NULL, NULL);
        or_f16_round_array(raw + L.wo_mlp[l].off, w16, (size_t)D * I);
        memset(st_b, 0, (size_t)2 * n * 4);
        or_emu_gemm(OR_RES | OR_STATS, m, w16, x, n, D, I, NULL, NULL, 0, NULL, NULL, st_b);
        if (trace_x)
            for (size_t i = 0; i < nD; i++) trace_x[(size_t)l * nD + i] = or_f32_from_f16(x[i]);
    }

    /* head input: st_a feeds in_proj and the scorer, st_b feeds linear1 */
    uint16_t *hx = malloc(nD * 2);
    or_emu_norm_add(x, raw + L.final_norm.off, raw + L.type_emb.off + (size_t)qtype * D, nh, D,
                    c->norm_eps, hx, st_a);
    if (head_trace)
        for (size_t i = 0; i < (size_t)nh * D; i++) head_trace[i] = or_f32_from_f16(hx[i]);
    for (int l = 0; l < c->n_head_layers; l++) {
        or_fold_layernorm_bias(raw + L.h_in_w[l].off, raw + L.h_norm1_w[l].off,
                               raw + L.h_norm1_b[l].off, raw + L.h_in_b[l].off, 3 * D, D, w16,
                               colsum, bias);
        or_emu_gemm(OR_LN | OR_BIAS, hx, w16, qkv, nh, 3 * D, D, st_a, colsum, c->head_eps, NULL,
                    bias, NULL);
        or_emu_attention(qkv, o, nh, H, 0);
        or_f16_round_array(raw + L.h_out_w[l].off, w16, (size_t)D * D);
        memset(st_b, 0, (size_t)2 * n * 4);
        or_emu_gemm(OR_BIAS | OR_RES | OR_STATS, o, w16, hx, nh, D, D, NULL, NULL, 0, NULL,
                    raw + L.h_out_b[l].off, st_b);
        or_fold_layernorm_bias(raw + L.h_l1_w[l].off, raw + L.h_norm2_w[l].off,
                               raw + L.h_norm2_b[l].off, raw + L.h_l1_b[l].off, F, D, w16, colsum,
                               bias);
        or_emu_gemm(OR_LN | OR_BIAS | OR_RELU, hx, w16, m, nh, F, D, st_b, colsum, c->head_eps,
                    NULL, bias, NULL);
        or_f16_round_array(raw + L.h_l2_w[l].off, w16, (size_t)D * F);
        memset(st_a, 0, (size_t)2 * n * 4);
        or_emu_gemm(OR_BIAS | OR_RES | OR_STATS, m, w16, hx, nh, D, F, NULL, NULL, 0, NULL,
                    raw + L.h_l2_b[l].off, st_a);
        if (head_trace)
            for (size_t i = 0; i < (size_t)nh * D; i++)
                head_trace[(size_t)(l + 1) * nh * D + i] = or_f32_from_f16(hx[i]);
    }
    or_fold_layernorm_bias(raw + L.s_lin1_w.off, raw + L.s_norm_w.off, raw + L.s_norm_b.off,
                           raw + L.s_lin1_b.off, S, D, w16, colsum, bias);
    or_emu_gemm(OR_LN | OR_BIAS | OR_GELU, hx, w16, y, nh, S, D, st_a, colsum, c->head_eps, NULL,
                bias, NULL);
    if (scorer_trace)
        for (int i = 0; i < n_markers; i++)
            for (int j = 0; j < S; j++)
                scorer_trace[(size_t)i * S + j] = or_f32_from_f16(y[(size_t)markers[i] * S + j]);
    uint16_t *w2 = malloc((size_t)S * 2);
    or_f16_round_array(raw + L.s_lin2_w.off, w2, (size_t)S);
    or_emu_score(y, w2, raw[L.s_lin2_b.off], markers, n_markers, S, logits);
    free(w2); free(hx);
    free(x); free(qkv); free(o); free(m); free(y); free(st_a); free(st_b); free(rg); free(rl);
    free(w16); free(colsum); free(bias); free(wtmp);
    return 0;
}

int or_forward_emu_head(const or_config *c, const float *raw, const uint32_t *ids, int n,
                        const uint32_t *markers, int n_markers, int qtype, int head_rows,
                        float *logits, float *trace_x, int bugs) {
    return or_forward_emu_full(c, raw, ids, n, markers, n_markers, qtype, head_rows, logits,
                               trace_x, NULL, NULL, bugs);
}

int or_forward_emu(const or_config *c, const float *raw, const uint32_t *ids, int n,
                   const uint32_t *markers, int n_markers, int qtype, float *logits,
                   float *trace_x, int bugs) {
    return or_forward_emu_head(c, raw, ids, n, markers, n_markers, qtype, 0, logits, trace_x,
                               bugs);
}
