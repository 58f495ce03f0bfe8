// The memory-bound kernels at the edges of the path: the token embedding with its LayerNorm, the
// head's input (final LayerNorm + question-type embedding, with row statistics), the marker-row
// gather, and the scorer's last D -> 1 product. One warp per row; rows are read with 8-byte
// vector loads and LayerNorm statistics are reduced with warp shuffles.
//
// Reference kernels: `embed` (kernels/src/main.rs:47-103), `norm_add` (:108-176), `score`
// (:180-200). Their width was fixed at 384; here it is a template parameter.
#pragma once
#include "common.cuh"

namespace jc {

// x[i] = LayerNorm(table[ids[i]]) * gamma (no bias), two-pass f32 statistics, f16 output; if
// stats is not null, also the row's sum and sum of squares of the stored values.
template <int D>
__global__ void __launch_bounds__(128) embed_kernel(const uint32_t *ids, uint32_t n,
                                                    const __half *table, const float *gamma,
                                                    float eps, __half *x, float *stats) {
    constexpr int PER = D / 128;  // 4-element chunks per lane
    const uint32_t row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (row >= n) return;
    const uint32_t id = ids[row];
    const uint2 *src = reinterpret_cast<const uint2 *>(table + (size_t)id * D);
    float v[PER * 4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        uint2 q = __ldg(src + j * 32 + lane);
        float2 a = unpack_half2(q.x), b = unpack_half2(q.y);
        v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = b.x; v[4 * j + 3] = b.y;
        sum += (a.x + a.y) + (b.x + b.y);
    }
    const float mean = warp_sum(sum) / D;
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < PER * 4; j++) var += (v[j] - mean) * (v[j] - mean);
    const float rstd = rsqrtf(warp_sum(var) / D + eps);
    uint2 *dst = reinterpret_cast<uint2 *>(x + (size_t)row * D);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    float s = 0.f, q2 = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const float4 gm = __ldg(g4 + j * 32 + lane);
        uint2 o;
        o.x = pack_half2((v[4 * j] - mean) * rstd * gm.x, (v[4 * j + 1] - mean) * rstd * gm.y);
        o.y = pack_half2((v[4 * j + 2] - mean) * rstd * gm.z, (v[4 * j + 3] - mean) * rstd * gm.w);
        dst[j * 32 + lane] = o;
        float2 a = unpack_half2(o.x), b = unpack_half2(o.y);
        s += (a.x + a.y) + (b.x + b.y);
        q2 += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
    }
    if (stats) {
        s = warp_sum(s);
        q2 = warp_sum(q2);
        if (lane == 0) {
            stats[2 * row] = s;
            stats[2 * row + 1] = q2;
        }
    }
}

// out[i] = LayerNorm(x[i]) * gamma + add (the encoder's final norm, then the question type's
// embedding), and each output row's sum and sum of squares of the stored values into stats.
template <int D>
__global__ void __launch_bounds__(128) norm_add_kernel(const __half *x, uint32_t n,
                                                       const float *gamma, const float *add,
                                                       float eps, __half *out, float *stats) {
    constexpr int PER = D / 128;
    const uint32_t row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (row >= n) return;
    const uint2 *src = reinterpret_cast<const uint2 *>(x + (size_t)row * D);
    float v[PER * 4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        uint2 q = src[j * 32 + lane];
        float2 a = unpack_half2(q.x), b = unpack_half2(q.y);
        v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = b.x; v[4 * j + 3] = b.y;
        sum += (a.x + a.y) + (b.x + b.y);
    }
    const float mean = warp_sum(sum) / D;
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < PER * 4; j++) var += (v[j] - mean) * (v[j] - mean);
    const float rstd = rsqrtf(warp_sum(var) / D + eps);
    uint2 *dst = reinterpret_cast<uint2 *>(out + (size_t)row * D);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    const float4 *a4 = reinterpret_cast<const float4 *>(add);
    float s = 0.f, q2 = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const float4 gm = __ldg(g4 + j * 32 + lane), ad = __ldg(a4 + j * 32 + lane);
        uint2 o;
        o.x = pack_half2((v[4 * j] - mean) * rstd * gm.x + ad.x,
                         (v[4 * j + 1] - mean) * rstd * gm.y + ad.y);
        o.y = pack_half2((v[4 * j + 2] - mean) * rstd * gm.z + ad.z,
                         (v[4 * j + 3] - mean) * rstd * gm.w + ad.w);
        dst[j * 32 + lane] = o;
        float2 a = unpack_half2(o.x), b = unpack_half2(o.y);
        s += (a.x + a.y) + (b.x + b.y);
        q2 += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
    }
    s = warp_sum(s);
    q2 = warp_sum(q2);
    if (lane == 0) {
        stats[2 * row] = s;
        stats[2 * row + 1] = q2;
    }
}

// out[i] = x[rows[i]] and its two statistics (one warp per gathered row).
__global__ void __launch_bounds__(128) gather_rows_kernel(const __half *x, const float *stats,
                                                          uint32_t d, const uint32_t *rows,
                                                          uint32_t k, uint32_t limit,
                                                          __half *out, float *out_stats,
                                                          unsigned int *err) {
    dev_err_bind(err);
    const uint32_t i = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (i >= k) return;
    const uint32_t r = rows[i];
    if (r >= limit) {
        // A marker past the rows the head computed: recorded, and the row is left unread.
        if (lane == 0) dev_fail(JC_DEV_BAD_INDEX);
        return;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)r * d);
    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)i * d);
    for (uint32_t j = lane; j < d / 8; j += 32) dst[j] = src[j];
    if (lane == 0) {
        out_stats[2 * i] = stats[2 * r];
        out_stats[2 * i + 1] = stats[2 * r + 1];
    }
}

// logits[i] = y[markers[i]] . w + b (one warp per marker; d even).
__global__ void __launch_bounds__(128) score_kernel(const __half *y, uint32_t d, const __half *w,
                                                    float b, const uint32_t *markers, uint32_t k,
                                                    float *logits) {
    const uint32_t i = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (i >= k) return;
    const uint32_t *row = reinterpret_cast<const uint32_t *>(y + (size_t)markers[i] * d);
    const uint32_t *wr = reinterpret_cast<const uint32_t *>(w);
    float acc = 0.f;
    for (uint32_t j = lane; j < d / 2; j += 32) {
        float2 a = unpack_half2(row[j]), c = unpack_half2(__ldg(wr + j));
        acc = fmaf(a.x, c.x, acc);
        acc = fmaf(a.y, c.y, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[i] = acc + b;
}

}  // namespace jc
