// Attention on the sm_100a tensor cores (tcgen05), for sequences long enough to fill 128-query
// tiles: o = softmax(q k^T / 8) v per 64-wide head, over all keys (global layers, the head) or
// keys with |q - k| <= window. Same semantics as attention.cuh (the reference's `attention` /
// `attention_task`, kernels/src/main.rs:303-542, and its key-range merge, kernels/src/attn.rs:
// 104-204); the f16 rounding of P and the f32 running sums are the same.
//
// A CTA takes 128 queries of one head and a range of 64-key tiles (the whole reach of its
// queries, or one of gridDim.z ranges of it, merged across CTAs in range order by the last to
// finish). Six warps:
//   - warp 4 lane 0 streams Q once and the K and V tiles of each key tile through a 3-deep ring
//     with TMA (qkv seen as (64 columns, rows, 3 x heads 64-column blocks), 128B swizzle, zero
//     fill past n; no multicast), and issues PV_j = P_j V_j (M 128, N 64 dims, K 64 keys, V read
//     MN-major straight from its TMA tile) into one of two TMEM buffers as soon as the softmax
//     has written P_j;
//   - warp 5 lane 0 issues S_j = Q K_j^T (M 128 queries, N 64 keys, K 64 dims) into one of two
//     more as soon as K_j has landed and the softmax has read S_{j-2}: the S and PV products are
//     two independent MMA chains;
//   - warps 0-3, one query row per thread (TMEM lane = row): read S_j from TMEM, mask, scale, keep
//     the running maximum and sum, write P_j = exp2(s - max) rounded to f16 into shared memory in
//     the 128B-swizzled K-major layout the MMA reads, then fold PV_{j-1} into f32 register
//     accumulators (o = o * alpha + PV), so no accumulator is rescaled in TMEM.
// The softmax threads' instruction issue bounds the loop, not the special-function unit's
// exponentials (half of them moved to a polynomial on the FMA pipe measured slower: 19.0 against
// 17.4 us for 1024 global tokens): the maximum and the sum are tree reductions and the scale rides
// in the exponent's FMA. Every wait is bounded (records a JC_DEV_TIMEOUT_* code and gives up).
#pragma once
#include "common.cuh"
#include "params.h"

namespace jc {

constexpr int ATC_QT = 128;      // queries per CTA (TMEM lanes)
constexpr int ATC_KT = 64;       // keys per tile
constexpr int ATC_STAGES = 3;    // K/V ring depth
constexpr int ATC_THREADS = 192;
constexpr int ATC_PART = 66;     // per-row partial of a key range: 64 accumulators, max, sum

// Shared memory, from a 1024-byte aligned base: Q | ring of (K, V) | two P tiles | barriers.
struct AtcSmem {
    static constexpr int TILE = 64 * 128;                  // 64 rows of 128 bytes
    static constexpr int Q = 0;                            // 128 rows
    static constexpr int KV = 2 * TILE;                    // stage s: K at KV + 2 s TILE, V after
    static constexpr int P = KV + ATC_STAGES * 2 * TILE;   // buffer b: 128 rows at P + 2 b TILE
    static constexpr int BAR = P + 2 * 2 * TILE;
    static constexpr int BYTES = BAR + 256;
    static constexpr int ALLOC = BYTES + 1024;             // + alignment slack
};

struct AttnTcParams {
    CUtensorMap map;  // qkv as (64, n, 3 heads), box (64, 64, 1)
    AttnParams p;
};

// Barrier among the 128 softmax threads (warps 0-3) only.
__device__ __forceinline__ void group_bar_atc() { asm volatile("bar.sync 1, 128;" ::: "memory"); }


// Descriptor of an MN-major operand tile whose K rows are 128 bytes (64 f16 along N), swizzled
// with the 128-byte pattern: stride byte offset = the next group of 8 K rows (1024 B); the leading
// byte offset (the next 64-wide N block) is never used at N = 64.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(8192 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__global__ void __launch_bounds__(ATC_THREADS, 2) attention_tc_kernel(const __grid_constant__ AttnTcParams kp) {
    dev_err_bind(kp.p.err);
    uint64_t *rec = threadIdx.x == 0 ? prof_record(kp.p.prof, kp.p.prof_cap) : nullptr;
    prof_open(rec);
    extern __shared__ uint8_t atc_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(atc_raw) + 1023) &
                                                ~uintptr_t(1023));
    const AttnParams &p = kp.p;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + AtcSmem::BAR);
    uint64_t *q_full = bars, *kv_full = bars + 1, *kv_empty = kv_full + ATC_STAGES;
    uint64_t *s_full = kv_empty + ATC_STAGES, *s_free = s_full + 2, *p_full = s_free + 2;
    uint64_t *pv_full = p_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pv_full + 2);
    uint32_t *last_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t q_tile = blockIdx.x, head = blockIdx.y, chunk = blockIdx.z, chunks = gridDim.z;
    const uint32_t n = p.n, window = p.window;
    // This CTA's query rows [q0, q_end): a 128-row tile, or a request-aligned entry of a packed
    // forward's tile list (written before the graph ran; an empty entry leaves at once).
    uint32_t q0 = q_tile * ATC_QT, q_end = min(q0 + ATC_QT, n);
    if (p.tiles) {
        const uint2 t = p.tiles[q_tile];
        q0 = t.x;
        q_end = min(t.y, n);
        if (q0 >= q_end || q_end - q0 > (uint32_t)ATC_QT) {
            if (threadIdx.x == 0 && q0 < q_end) dev_fail(JC_DEV_BAD_INDEX);
            return;
        }
    }

    // The key tiles some query of this CTA can reach (the spans of its first and last query
    // bound the others'), and this CTA's range of them.
    int lo_first, hi_first, lo_last, hi_last;
    key_span(p.seg, n, window, q0, lo_first, hi_first);
    key_span(p.seg, n, window, q_end - 1, lo_last, hi_last);
    const uint32_t kb_lo = (uint32_t)max(lo_first, 0) / ATC_KT;
    const uint32_t kb_hi = (uint32_t)max(hi_last, lo_first) / ATC_KT + 1;
    const uint32_t span = kb_hi - kb_lo;
    const uint32_t kb0 = kb_lo + chunk * span / chunks;
    const uint32_t T = kb_lo + (chunk + 1) * span / chunks - kb0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ATC_STAGES; s++) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 2);  // the S and the PV issuer each release a stage
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_free[b], 4);
            mbar_init(&p_full[b], 4);
            mbar_init(&pv_full[b], 1);
        }
        fence_barrier_init();
    }
    if (warp == 5) tmem_alloc(tmem_slot, 256);
    if (threadIdx.x == 128) tma_prefetch_desc(&kp.map);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // columns: S 0 / 64, PV 128 / 192
    pdl_wait();
    pdl_launch_dependents();
    prof_stamp(rec, 1);

    if (warp == 4) {
        if (lane == 0 && T > 0) {
            const int32_t hq = (int32_t)head, hk = (int32_t)(p.heads + head),
                          hv = (int32_t)(2 * p.heads + head);
            auto load_kv = [&](uint32_t j) {
                const uint32_t s = j % ATC_STAGES;
                uint8_t *st = base + AtcSmem::KV + s * 2 * AtcSmem::TILE;
                mbar_arrive_expect_tx(&kv_full[s], 2 * AtcSmem::TILE);
                const int32_t k0 = (int32_t)((kb0 + j) * ATC_KT);
                tma_load_3d(st, &kp.map, &kv_full[s], 0, k0, hk);
                tma_load_3d(st + AtcSmem::TILE, &kp.map, &kv_full[s], 0, k0, hv);
            };
            mbar_arrive_expect_tx(q_full, 2 * AtcSmem::TILE);
            tma_load_3d(base + AtcSmem::Q, &kp.map, q_full, 0, (int32_t)q0, hq);
            tma_load_3d(base + AtcSmem::Q + AtcSmem::TILE, &kp.map, q_full, 0, (int32_t)q0 + 64, hq);
            uint32_t issued = 0;
            for (; issued < T && issued < (uint32_t)ATC_STAGES; issued++) load_kv(issued);
            constexpr uint32_t idesc_o = umma_idesc_f16(ATC_QT, 64) | (1u << 16);  // B (V) MN-major
            for (uint32_t j = 0; j < T; j++) {
                const uint32_t b = j & 1, s = j % ATC_STAGES;
                // P_j written (every softmax thread had folded PV_{j-2}, whose buffer PV_j reuses,
                // before writing it) and V_j landed.
                if (!mbar_wait(&p_full[b], (j >> 1) & 1, JC_DEV_TIMEOUT_FULL) ||
                    !mbar_wait(&kv_full[s], (j / ATC_STAGES) & 1, JC_DEV_TIMEOUT_FULL))
                    break;
                tc_fence_after();
                const uint32_t p_a = smem_u32(base + AtcSmem::P + b * 2 * AtcSmem::TILE);
                const uint32_t v_a = smem_u32(base + AtcSmem::KV + s * 2 * AtcSmem::TILE + AtcSmem::TILE);
#pragma unroll
                for (uint32_t kk = 0; kk < 4; kk++)
                    // P: +32 bytes per 16 keys inside its 128-byte rows; V: +16 rows of 128 bytes.
                    tc_mma_f16(tmem + 128 + b * 64, umma_desc_sw128(p_a) + 2 * kk,
                               umma_desc_sw128_mn(v_a + kk * 2048), idesc_o, kk > 0);
                tc_commit(&pv_full[b]);
                tc_commit(&kv_empty[s]);
                // Stage s takes tile j + STAGES once both products of tile j have read it.
                if (issued < T) {
                    if (!mbar_wait(&kv_empty[s], (j / ATC_STAGES) & 1, JC_DEV_TIMEOUT_EMPTY)) break;
                    load_kv(issued++);
                }
            }
            // No copy may land after the CTA has left: wait (bounded) for the last ones.
            mbar_wait(q_full, 0, JC_DEV_TIMEOUT_FULL);
            for (uint32_t j = issued > (uint32_t)ATC_STAGES ? issued - ATC_STAGES : 0; j < issued; j++)
                mbar_wait(&kv_full[j % ATC_STAGES], (j / ATC_STAGES) & 1, JC_DEV_TIMEOUT_FULL);
        }
    } else if (warp == 5) {
        if (lane == 0 && T > 0) {
            constexpr uint32_t idesc_s = umma_idesc_f16(ATC_QT, ATC_KT);
            const uint32_t q_a = smem_u32(base + AtcSmem::Q);
            bool ok = mbar_wait(q_full, 0, JC_DEV_TIMEOUT_FULL);
            for (uint32_t j = 0; ok && j < T; j++) {
                const uint32_t b = j & 1, s = j % ATC_STAGES;
                if (!mbar_wait(&kv_full[s], (j / ATC_STAGES) & 1, JC_DEV_TIMEOUT_FULL) ||
                    (j >= 2 && !mbar_wait(&s_free[b], ((j - 2) >> 1) & 1, JC_DEV_TIMEOUT_EMPTY)))
                    break;
                tc_fence_after();
                const uint32_t k_a = smem_u32(base + AtcSmem::KV + s * 2 * AtcSmem::TILE);
#pragma unroll
                for (uint32_t kk = 0; kk < 4; kk++)
                    tc_mma_f16(tmem + b * 64, umma_desc_sw128(q_a) + 2 * kk,
                               umma_desc_sw128(k_a) + 2 * kk, idesc_s, kk > 0);
                tc_commit(&s_full[b]);
                tc_commit(&kv_empty[s]);
            }
        }
    } else {
        // Softmax: thread = query row of the tile = TMEM lane.
        const uint32_t row = threadIdx.x, q = q0 + row;
        const uint32_t lane_base = tmem + ((warp * 32) << 16);
        // This row's key span, and the keys every row of the warp sees.
        int row_lo, row_hi, w_lo, w_hi, unused;
        key_span(p.seg, n, window, q, row_lo, row_hi);
        key_span(p.seg, n, window, q0 + warp * 32 + 31, w_lo, unused);
        key_span(p.seg, n, window, q0 + warp * 32, unused, w_hi);
        const float scale = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
        float o[64];
#pragma unroll
        for (int e = 0; e < 64; e++) o[e] = 0.f;
        float mx = -INFINITY, lsum = 0.f, alpha_prev = 1.f;
        bool ok = true;
        auto fold = [&](uint32_t i, float a) -> bool {
            const uint32_t b = i & 1;
            if (!mbar_wait(&pv_full[b], (i >> 1) & 1, JC_DEV_TIMEOUT_MMA)) return false;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; h++) {  // in halves: 32 more registers, not 64
                float v[32];
                tmem_ld<16>(lane_base + 128 + b * 64 + 32 * h, v);
                tmem_ld<16>(lane_base + 128 + b * 64 + 32 * h + 16, v + 16);
                tc_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; e++) o[32 * h + e] = fmaf(o[32 * h + e], a, v[e]);
            }
            tc_fence_before();
            return true;
        };
        for (uint32_t j = 0; j < T; j++) {
            const uint32_t b = j & 1;
            float alpha = 1.f;
            if (ok) ok = mbar_wait(&s_full[b], (j >> 1) & 1, JC_DEV_TIMEOUT_MMA);
            if (ok) {
                tc_fence_after();
                float sc[64];
                tmem_ld<16>(lane_base + b * 64, sc);
                tmem_ld<16>(lane_base + b * 64 + 16, sc + 16);
                tmem_ld<16>(lane_base + b * 64 + 32, sc + 32);
                tmem_ld<16>(lane_base + b * 64 + 48, sc + 48);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[b]);

                // Mask (unless every key of the tile is visible to every row of this warp), then
                // the tile's maximum in a tree (the scale is positive: max(s) * scale is the
                // maximum of the scaled scores).
                const uint32_t k0 = (kb0 + j) * ATC_KT;
                const bool interior = (int)k0 >= w_lo && (int)k0 + ATC_KT - 1 <= w_hi;
                if (!interior) {
                    // This row sees keys [row_lo, row_hi]: columns [clo, chi) of the tile.
                    const int clo = row_lo - (int)k0, chi = row_hi - (int)k0 + 1;
#pragma unroll
                    for (int c = 0; c < 64; c++) sc[c] = (c >= clo && c < chi) ? sc[c] : -INFINITY;
                }
                float m8[8];
#pragma unroll
                for (int c = 0; c < 8; c++) m8[c] = fmaxf(sc[c], sc[c + 8]);
#pragma unroll
                for (int c = 16; c < 64; c++) m8[c & 7] = fmaxf(m8[c & 7], sc[c]);
                const float mt = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale;
                const float m_new = fmaxf(mx, mt);
                const float bse = m_new == -INFINITY ? 0.f : m_new;
                alpha = ex2_approx(mx - bse);
                mx = m_new;
                // P row into the K-major 128B-swizzled tile, a 16-byte chunk (8 keys) at a time:
                // chunk c at chunk c ^ (row % 8).
                uint8_t *prow = base + AtcSmem::P + b * 2 * AtcSmem::TILE + row * 128;
                float r8[8];
#pragma unroll
                for (uint32_t c = 0; c < 8; c++) {
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float a0 = ex2_approx(fmaf(sc[8 * c + 2 * e], scale, -bse));
                        const float a1 = ex2_approx(fmaf(sc[8 * c + 2 * e + 1], scale, -bse));
                        r8[2 * (e & 1) + (c & 1) * 4 + (e >> 1)] =
                            c < 2 ? a0 + a1 : r8[2 * (e & 1) + (c & 1) * 4 + (e >> 1)] + (a0 + a1);
                        pk[e] = pack_half2(a0, a1);
                    }
                    *reinterpret_cast<uint4 *>(prow + ((c ^ (row & 7)) << 4)) =
                        make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                lsum = lsum * alpha + (((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7])));
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
            }
            if (j >= 1 && ok) ok = fold(j - 1, alpha_prev);
            alpha_prev = alpha;
        }
        if (ok && T > 0) ok = fold(T - 1, alpha_prev);

        const uint32_t D = p.heads * 64;
        if (chunks > 1) {
            // This range's partial, stored [value][row] so the stores coalesce; the last range of
            // the (query tile, head) to finish merges every range in range order.
            const uint32_t tile = q_tile * p.heads + head;
            float *slot = p.ws + ((size_t)tile * chunks + chunk) * ATC_PART * ATC_QT + row;
#pragma unroll
            for (int e = 0; e < 64; e++) slot[e * ATC_QT] = o[e];
            slot[64 * ATC_QT] = mx;
            slot[65 * ATC_QT] = lsum;
            __threadfence();
            group_bar_atc();
            if (row == 0) {
                const uint32_t old = atomicAdd(&p.counters[tile], 1u);
                const bool last = old == chunks - 1;
                if (last) p.counters[tile] = 0;
                *last_flag = last ? 1u : 0u;
            }
            group_bar_atc();
            if (*last_flag) {
                __threadfence();
                const float *base_slot = p.ws + (size_t)tile * chunks * ATC_PART * ATC_QT + row;
                float m2 = -INFINITY;
                for (uint32_t zz = 0; zz < chunks; zz++)
                    m2 = fmaxf(m2, __ldcg(base_slot + ((size_t)zz * ATC_PART + 64) * ATC_QT));
                const float bm = m2 == -INFINITY ? 0.f : m2;
#pragma unroll
                for (int e = 0; e < 64; e++) o[e] = 0.f;
                lsum = 0.f;
                for (uint32_t zz = 0; zz < chunks; zz++) {
                    const float *sl = base_slot + (size_t)zz * ATC_PART * ATC_QT;
                    const float f = exp2f(__ldcg(sl + 64 * ATC_QT) - bm);
                    lsum += __ldcg(sl + 65 * ATC_QT) * f;
#pragma unroll
                    for (int e = 0; e < 64; e++) o[e] += __ldcg(sl + e * ATC_QT) * f;
                }
            } else {
                ok = false;  // another range stores the rows
            }
        }
        if (ok && q < q_end) {
            const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
            uint4 *dst = reinterpret_cast<uint4 *>(p.o + (size_t)q * D + head * 64);
#pragma unroll
            for (int c = 0; c < 8; c++)
                dst[c] = make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv),
                                    pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                                    pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                                    pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
        }
    }
    // Every TMEM read and MMA is done before the columns are freed.
    tc_fence_before();
    __syncthreads();
    prof_stamp(rec, 4);
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
    prof_stamp(rec, 5);
}

}  // namespace jc
