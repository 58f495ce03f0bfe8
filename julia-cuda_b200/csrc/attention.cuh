// Attention for the encoder and the head: o = softmax(q k^T / 8) v per 64-wide head, over all keys
// (global layers, the head) or keys with |q - k| <= window (sliding-window layers).
//
// Replaces the reference's `attention` / `attention_task` (kernels/src/main.rs:303-542) and its
// key-range merge (kernels/src/attn.rs:104-204). FlashAttention-2 structure with the key loop
// split inside the CTA: a CTA takes 16 * QW queries of one head and runs QW x KS warps; warp group
// g (QW warps, 16 queries each) streams key tiles g, g + KS, g + 2 KS, ... of the CTA's key range
// through its own double-buffered, XOR-swizzled shared-memory slots with cp.async, keeping S and
// the running max / sum in registers (online softmax in exp2 on the special-function unit),
// rounding P to f16 for the P.V product and O in f32. The KS partial results meet in shared
// memory and are merged in group order, so the output does not depend on timing. Sequences of a
// few hundred tokens therefore run at most a couple of dependent key-tile steps per warp.
// d = 64 tiles are too small for 128-row tcgen05 tiles at these lengths, so the products use
// the 16x8x16 tensor-core MMA.
//
// Sliding-window CTAs only visit the key tiles some query of theirs can reach. For long global
// sequences the key range can also be split across CTAs (gridDim.z ranges): each range stores
// its partial, and the last range of a (query tile, head) to finish (atomic counter, reset by it)
// merges all of them in range order.
//
// qkv rows are [q | k | v], each `heads` heads of 64, in natural (checkpoint) order.
#pragma once
#include "common.cuh"
#include "params.h"

namespace jc {

// Swizzled [rows][64] f16 tile: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
__device__ __forceinline__ uint32_t swz64_off(uint32_t row, uint32_t chunk) {
    return row * 64 + ((chunk ^ (row & 7)) << 3);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool pred) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(pred ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Barrier among the `count` threads of one warp group (named barrier `id`, 1..15).
__device__ __forceinline__ void group_bar(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// c += a (16x16, row) * b (16x8, col), f16 inputs, f32 accumulators.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Rows [row0, row0 + ROWS) of one head of one third (0 q, 1 k, 2 v) into a swizzled tile by the
// `nthreads` threads of a group (thread index t); rows past n are zero-filled.
template <int ROWS>
__device__ __forceinline__ void load_head_tile(uint32_t tile, const AttnParams &p, uint32_t row0,
                                               uint32_t head, uint32_t third, uint32_t t,
                                               uint32_t nthreads) {
    const uint32_t D = p.heads * 64;
    for (uint32_t c = t; c < ROWS * 8; c += nthreads) {
        const uint32_t row = c >> 3, ch = c & 7;
        const uint32_t r = row0 + row;
        const bool ok = r < p.n;
        const __half *src = p.qkv + (size_t)(ok ? r : 0) * 3 * D + third * D + head * 64 + ch * 8;
        cp_async16(tile + swz64_off(row, ch) * 2, src, ok);
    }
}

constexpr int ATTN_PART = 36;  // per-thread partial: 32 accumulators, 2 maxima, 2 sums

template <int QW, int KS>
struct AttnShape {
    static constexpr int QT = 16 * QW;
    static constexpr int THREADS = 32 * QW * KS;
    static constexpr int GT = 32 * QW;  // threads per key group
    static constexpr int SLOT = 2 * 64 * 64 * 2;  // K and V tile of 64 keys, bytes
    static constexpr int SMEM = QT * 64 * 2 + KS * 2 * SLOT + 128;
    static_assert((KS - 1) * ATTN_PART * GT * 4 <= KS * 2 * SLOT, "partials must fit the slots");
};

// One (query tile, head, key range) task; every thread of the CTA calls it. `smem`: the task's
// shared memory (AttnShape::SMEM bytes, 128-byte aligned). `standalone`: the single-attention
// kernel (programmatic dependent launch waits here); in the persistent kernel a grid barrier has
// already ordered the inputs.
template <int QW, int KS>
__device__ __forceinline__ void attention_task(const AttnParams &p, uint8_t *smem, uint32_t q_tile,
                                               uint32_t head, uint32_t chunk, uint32_t chunks,
                                               bool standalone) {
    using S = AttnShape<QW, KS>;
    constexpr int QT = S::QT, GT = S::GT;
    __half *qs = reinterpret_cast<__half *>(smem);
    uint8_t *slots = smem + QT * 64 * 2;
    uint32_t *last_flag = reinterpret_cast<uint32_t *>(slots + KS * 2 * S::SLOT);

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t grp = warp / QW, qw = warp % QW, tg = threadIdx.x % GT;
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t q0 = q_tile * QT;
    const uint32_t n = p.n, window = p.window;

    // Key tiles some query of this CTA can reach (the spans of its first and last query bound
    // those of the others), this CTA's range of them, this group's share.
    int lo_first, hi_first, lo_last, hi_last;
    key_span(p.seg, n, window, q0, lo_first, hi_first);
    key_span(p.seg, n, window, min(q0 + QT - 1, n - 1), lo_last, hi_last);
    const uint32_t kb_lo = (uint32_t)max(lo_first, 0) / 64;
    const uint32_t kb_hi = (uint32_t)max(hi_last, lo_first) / 64 + 1;
    const uint32_t span = kb_hi - kb_lo;
    const uint32_t kb0 = kb_lo + chunk * span / chunks, kb1 = kb_lo + (chunk + 1) * span / chunks;
    const uint32_t my_n = kb1 > kb0 + grp ? (kb1 - kb0 - grp + KS - 1) / KS : 0;

    uint64_t *rec = threadIdx.x == 0 ? prof_record(p.prof, p.prof_cap) : nullptr;
    if (standalone) {
        pdl_wait();
        pdl_launch_dependents();
    }
    prof_stamp(rec, 1);
    __syncthreads();  // the previous task of this CTA is done with the shared memory

    const uint32_t qs_a = smem_u32(qs);
    const uint32_t slot_a = smem_u32(slots) + grp * 2 * S::SLOT;
    auto kb_of = [&](uint32_t j) { return kb0 + grp + j * KS; };

    load_head_tile<QT>(qs_a, p, q0, head, 0, threadIdx.x, S::THREADS);
    if (my_n > 0) {
        load_head_tile<64>(slot_a, p, kb_of(0) * 64, head, 1, tg, GT);
        load_head_tile<64>(slot_a + S::SLOT / 2, p, kb_of(0) * 64, head, 2, tg, GT);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    prof_stamp(rec, 2);

    uint32_t qf[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; kk++)
        ldsm_x4(qs_a + swz64_off(qw * 16 + (lane & 15), kk * 2 + (lane >> 4)) * 2, qf[kk][0],
                qf[kk][1], qf[kk][2], qf[kk][3]);

    const float scale = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
    const uint32_t qrow[2] = {q0 + qw * 16 + g, q0 + qw * 16 + g + 8};
    // This lane's two rows' key spans, and the keys every row of the warp sees.
    int row_lo[2], row_hi[2], w_lo, w_hi, unused;
    key_span(p.seg, n, window, qrow[0], row_lo[0], row_hi[0]);
    key_span(p.seg, n, window, qrow[1], row_lo[1], row_hi[1]);
    key_span(p.seg, n, window, q0 + qw * 16 + 15, w_lo, unused);
    key_span(p.seg, n, window, q0 + qw * 16, unused, w_hi);
    float mx[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (uint32_t j = 0; j < my_n; j++) {
        const uint32_t buf = j & 1;
        if (j + 1 < my_n) {
            const uint32_t nxt = slot_a + (buf ^ 1) * S::SLOT;
            load_head_tile<64>(nxt, p, kb_of(j + 1) * 64, head, 1, tg, GT);
            load_head_tile<64>(nxt + S::SLOT / 2, p, kb_of(j + 1) * 64, head, 2, tg, GT);
        }
        cp_async_commit();
        cp_async_wait<1>();
        group_bar(1 + grp, GT);
        const uint32_t ks_a = slot_a + buf * S::SLOT, vs_a = ks_a + S::SLOT / 2;

        // S = Q K^T: 16 queries x 64 keys per warp (8 n-tiles of 8 keys).
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
#pragma unroll
            for (int jp = 0; jp < 4; jp++) {
                const uint32_t mi = lane >> 3;
                const uint32_t key = jp * 16 + (mi >> 1) * 8 + (lane & 7);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(ks_a + swz64_off(key, kk * 2 + (mi & 1)) * 2, b0, b1, b2, b3);
                mma16816(s[2 * jp], qf[kk], b0, b1);
                mma16816(s[2 * jp + 1], qf[kk], b2, b3);
            }
        }

        // Mask, scale and the online softmax. Row h of this lane: elements 2h, 2h+1 of each tile.
        // A tile every key of which every query of this warp may see (inside the spans of the
        // warp's first and last query, which bound the others') needs no mask.
        const uint32_t k0 = kb_of(j) * 64;
        const bool interior = (int)k0 >= w_lo && (int)k0 + 63 <= w_hi;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float m = -INFINITY;
            if (interior) {
#pragma unroll
                for (int jt = 0; jt < 8; jt++)
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const float v = s[jt][2 * h + e] * scale;
                        s[jt][2 * h + e] = v;
                        m = fmaxf(m, v);
                    }
            } else {
#pragma unroll
                for (int jt = 0; jt < 8; jt++)
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int key = (int)(k0 + 8 * jt + 2 * t + e);
                        const bool ok = key >= row_lo[h] && key <= row_hi[h];
                        const float v = ok ? s[jt][2 * h + e] * scale : -INFINITY;
                        s[jt][2 * h + e] = v;
                        m = fmaxf(m, v);
                    }
            }
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            const float m_new = fmaxf(mx[h], m);
            const float base = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = ex2_approx(mx[h] - base);
            mx[h] = m_new;
            float rs = 0.f;
#pragma unroll
            for (int jt = 0; jt < 8; jt++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float pv = ex2_approx(s[jt][2 * h + e] - base);
                    s[jt][2 * h + e] = pv;
                    rs += pv;
                }
                acc[jt][2 * h] *= alpha;
                acc[jt][2 * h + 1] *= alpha;
            }
            lsum[h] = lsum[h] * alpha + rs;
        }

        // O += P V: P (rounded to f16) as the A operand, V through ldmatrix.trans.
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t a[4];
            a[0] = pack_half2(s[2 * kk][0], s[2 * kk][1]);
            a[1] = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            a[2] = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            a[3] = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {
                const uint32_t mi = lane >> 3;
                const uint32_t key = kk * 16 + (mi & 1) * 8 + (lane & 7);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vs_a + swz64_off(key, dp * 2 + (mi >> 1)) * 2, b0, b1, b2, b3);
                mma16816(acc[2 * dp], a, b0, b1);
                mma16816(acc[2 * dp + 1], a, b2, b3);
            }
        }
        group_bar(1 + grp, GT);
    }
    cp_async_wait<0>();
    prof_stamp(rec, 3);

    // The key groups' partials meet in shared memory (the slots are free now), merged in group
    // order by group 0.
    if constexpr (KS > 1) {
        __syncthreads();
        float *part = reinterpret_cast<float *>(slots);
        if (grp > 0) {
            float *my = part + (size_t)(grp - 1) * ATTN_PART * GT + tg;
#pragma unroll
            for (int jt = 0; jt < 8; jt++)
#pragma unroll
                for (int e = 0; e < 4; e++) my[(jt * 4 + e) * GT] = acc[jt][e];
            my[32 * GT] = mx[0];
            my[33 * GT] = mx[1];
            my[34 * GT] = lsum[0];
            my[35 * GT] = lsum[1];
        }
        __syncthreads();
        if (grp == 0) {
            float m2[2] = {mx[0], mx[1]};
#pragma unroll
            for (int gg = 1; gg < KS; gg++) {
                const float *o = part + (size_t)(gg - 1) * ATTN_PART * GT + tg;
                m2[0] = fmaxf(m2[0], o[32 * GT]);
                m2[1] = fmaxf(m2[1], o[33 * GT]);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float b = m2[h] == -INFINITY ? 0.f : m2[h];
                const float f0 = exp2f(mx[h] - b);
                lsum[h] *= f0;
#pragma unroll
                for (int jt = 0; jt < 8; jt++) {
                    acc[jt][2 * h] *= f0;
                    acc[jt][2 * h + 1] *= f0;
                }
#pragma unroll
                for (int gg = 1; gg < KS; gg++) {
                    const float *o = part + (size_t)(gg - 1) * ATTN_PART * GT + tg;
                    const float f = exp2f(o[(32 + h) * GT] - b);
                    lsum[h] += o[(34 + h) * GT] * f;
#pragma unroll
                    for (int jt = 0; jt < 8; jt++) {
                        acc[jt][2 * h] += o[(jt * 4 + 2 * h) * GT] * f;
                        acc[jt][2 * h + 1] += o[(jt * 4 + 2 * h + 1) * GT] * f;
                    }
                }
                mx[h] = m2[h];
            }
        }
    }
    if (grp != 0) return;

    if (chunks > 1) {
        // Partial of this CTA's key range, stored [value][thread] so the stores coalesce; the
        // last range of the (query tile, head) merges all of them in range order.
        const uint32_t tile = q_tile * p.heads + head;
        float *slot = p.ws + ((size_t)tile * chunks + chunk) * ATTN_PART * GT + tg;
#pragma unroll
        for (int jt = 0; jt < 8; jt++)
#pragma unroll
            for (int e = 0; e < 4; e++) slot[(jt * 4 + e) * GT] = acc[jt][e];
        slot[32 * GT] = mx[0];
        slot[33 * GT] = mx[1];
        slot[34 * GT] = lsum[0];
        slot[35 * GT] = lsum[1];
        __threadfence();
        group_bar(1, GT);
        if (tg == 0) {
            const uint32_t old = atomicAdd(&p.counters[tile], 1u);
            const bool last = old == chunks - 1;
            if (last) p.counters[tile] = 0;
            *last_flag = last ? 1u : 0u;
        }
        group_bar(1, GT);
        if (!*last_flag) return;
        __threadfence();
        const float *base_slot = p.ws + (size_t)tile * chunks * ATTN_PART * GT + tg;
        float m2[2] = {-INFINITY, -INFINITY};
        for (uint32_t zz = 0; zz < chunks; zz++) {
            const float *sl = base_slot + (size_t)zz * ATTN_PART * GT;
            m2[0] = fmaxf(m2[0], __ldcg(sl + 32 * GT));
            m2[1] = fmaxf(m2[1], __ldcg(sl + 33 * GT));
        }
#pragma unroll
        for (int jt = 0; jt < 8; jt++) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.f;
        lsum[0] = lsum[1] = 0.f;
        for (uint32_t zz = 0; zz < chunks; zz++) {
            const float *sl = base_slot + (size_t)zz * ATTN_PART * GT;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float b = m2[h] == -INFINITY ? 0.f : m2[h];
                const float f = exp2f(__ldcg(sl + (32 + h) * GT) - b);
                lsum[h] += __ldcg(sl + (34 + h) * GT) * f;
#pragma unroll
                for (int jt = 0; jt < 8; jt++) {
                    acc[jt][2 * h] += __ldcg(sl + (jt * 4 + 2 * h) * GT) * f;
                    acc[jt][2 * h + 1] += __ldcg(sl + (jt * 4 + 2 * h + 1) * GT) * f;
                }
            }
        }
    }

    const uint32_t D = p.heads * 64;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float l = lsum[h];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        if (qrow[h] < n) {
            uint32_t *dst = reinterpret_cast<uint32_t *>(p.o + (size_t)qrow[h] * D + head * 64);
#pragma unroll
            for (int jt = 0; jt < 8; jt++)
                dst[(8 * jt + 2 * t) / 2] = pack_half2(acc[jt][2 * h] * inv, acc[jt][2 * h + 1] * inv);
        }
    }
    prof_stamp(rec, 4);
}

// Two CTAs per SM (at most 128 registers a thread), so the 64-query shape's grid at 1024 tokens
// (16 query tiles x 12 heads) is resident in one wave; five key groups (320 threads, 164 KB of
// shared memory) fit one CTA an SM whatever the registers, so they are not capped.
template <int QW, int KS>
__global__ void __launch_bounds__(32 * QW * KS, KS > 4 ? 1 : 2) attention_kernel(const AttnParams p) {
    dev_err_bind(p.err);
    uint64_t *rec = threadIdx.x == 0 ? prof_record(p.prof, p.prof_cap) : nullptr;
    prof_open(rec);
    extern __shared__ __align__(128) uint8_t att_smem[];
    attention_task<QW, KS>(p, att_smem, blockIdx.x, blockIdx.y, blockIdx.z, gridDim.z, true);
    prof_stamp(rec, 5);
}

}  // namespace jc
