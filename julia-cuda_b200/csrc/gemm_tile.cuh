// One GEMM output tile as a device function (the body of both the single-GEMM kernel and of the
// persistent kernel's GEMM phases), its set-up / tear-down, and the single-GEMM kernel.
#pragma once
#include "gemm.cuh"

namespace jc {

// Where a CTA's GEMM pipeline lives in shared memory: STAGES stages, then the tail: the barriers,
// the TMEM base slot, a flag, per-row partial statistics and the tile's column sums / biases. The
// tail normally follows the stages; a CTA that runs tiles of two widths (the persistent kernel)
// places both views' tails at one offset past the larger stage area, their barriers bar_off bytes
// apart inside it.
template <int BN, int STAGES, int BM = GEMM_BM>
struct GemmSmemView {
    using S = GemmShape<BN, STAGES, BM>;
    uint8_t *stages;
    uint64_t *full, *empty, *done, *recv_bar;
    uint32_t *tmem_slot, *last_flag;
    float2 *row_part;
    float *cs_s, *bs_s;
    float *recv;  // cluster split-K partials from the peers (S::RECV_BYTES<CS>, after the tail)
    __device__ explicit GemmSmemView(uint8_t *base, uint32_t tail_at = STAGES * S::STAGE_BYTES,
                                     uint32_t bar_off = 0) {
        stages = base;
        uint8_t *tail = base + tail_at;
        full = reinterpret_cast<uint64_t *>(tail + bar_off);
        empty = full + STAGES;
        done = empty + STAGES;
        recv_bar = done + 1;
        tmem_slot = reinterpret_cast<uint32_t *>(recv_bar + 1);
        last_flag = tmem_slot + 1;
        row_part = reinterpret_cast<float2 *>(tail + 256);
        cs_s = reinterpret_cast<float *>(tail + 256 + 1024);
        bs_s = cs_s + BN;
        recv = reinterpret_cast<float *>(tail + S::TAIL_BYTES);
    }
};

// A CTA's pipeline position across tiles (every thread keeps the same copy): stages filled so far
// (slot = it % STAGES, ring round = it / STAGES) and tiles finished (the accumulator barrier's
// parity).
struct GemmRun {
    uint32_t it = 0;
    uint32_t tiles = 0;
};

// A view's barriers (thread 0; the caller's next CTA barrier publishes them).
template <int BN, int STAGES, int BM = GEMM_BM>
__device__ __forceinline__ void gemm_init_barriers(const GemmSmemView<BN, STAGES, BM> &sv) {
    constexpr uint32_t NI = GemmShape<BN, STAGES>::NI;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&sv.full[s], 1);
            mbar_init(&sv.empty[s], NI);  // every issuer releases every stage
        }
        mbar_init(sv.done, NI);
        fence_barrier_init();
    }
}

// Barrier initialisation and the TMEM accumulator; every thread calls it, returns the TMEM base.
template <int BN, int STAGES, int BM = GEMM_BM>
__device__ __forceinline__ uint32_t gemm_setup(const GemmSmemView<BN, STAGES, BM> &sv) {
    gemm_init_barriers<BN, STAGES, BM>(sv);
    if ((threadIdx.x >> 5) == 0) tmem_alloc(sv.tmem_slot, GemmShape<BN, STAGES>::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return *sv.tmem_slot;
}

template <int BN, int STAGES>
__device__ __forceinline__ void gemm_teardown(uint32_t tmem) {
    tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, GemmShape<BN, STAGES>::TMEM_COLS);
    }
}

// Stages a range of nkb k-blocks takes.
__device__ __forceinline__ uint32_t gemm_stages(uint32_t nkb) { return (nkb + GEMM_KPS - 1) / GEMM_KPS; }

// Producer thread only: the W half of stages [first, count) of a tile whose pipeline starts at
// run.it and whose k range starts at k-block kb0 (expect_tx covers A and W; the A halves follow
// once the activations are ready). A stage's box may reach past the range (or past k): those
// k-blocks are loaded (zeros past k) but never multiplied.
template <int BN, int STAGES, int BM = GEMM_BM>
__device__ __forceinline__ bool gemm_issue_w(const GemmParams &p,
                                             const GemmSmemView<BN, STAGES, BM> &sv,
                                             uint32_t it, uint32_t n0, uint32_t kb0,
                                             uint32_t first, uint32_t count) {
    using S = GemmShape<BN, STAGES, BM>;
    for (uint32_t i = first; i < count; i++) {
        const uint32_t g = it + i, s = g % STAGES, round = g / STAGES;
        if (round > 0 && !mbar_wait(&sv.empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY))
            return false;
        uint8_t *st = sv.stages + s * S::STAGE_BYTES;
        mbar_arrive_expect_tx(&sv.full[s], S::STAGE_BYTES);
        tma_load_3d(st + S::A_BYTES, p.map_w, &sv.full[s], 0, (int32_t)n0,
                    (int32_t)(kb0 + i * GEMM_KPS));
    }
    return true;
}

// Producer thread only: the A half of stage i (whose W half and expect_tx are already issued).
template <int BN, int STAGES, int BM = GEMM_BM>
__device__ __forceinline__ void gemm_issue_a(const GemmParams &p,
                                             const GemmSmemView<BN, STAGES, BM> &sv,
                                             uint32_t it, uint32_t m0, uint32_t kb0, uint32_t i) {
    using S = GemmShape<BN, STAGES, BM>;
    const uint32_t s = (it + i) % STAGES;
    tma_load_3d(sv.stages + s * S::STAGE_BYTES, p.map_a, &sv.full[s], 0, (int32_t)m0,
                (int32_t)(kb0 + i * GEMM_KPS));
}

// v[0, G) = columns [ta, ta + G) and v[G, 2G) = columns [tb, tb + G) of this thread's TMEM lane,
// each summed over the NI accumulators (BN columns apart) in accumulator order, so the result does
// not depend on timing. Every accumulator's columns are requested before the one wait.
template <int G, int NI, int BN>
__device__ __forceinline__ void acc_ld2(uint32_t ta, uint32_t tb, float *v) {
    tmem_ld<G>(ta, v);
    tmem_ld<G>(tb, v + G);
    if constexpr (NI > 1) {
        float t[NI - 1][2 * G];
#pragma unroll
        for (int j = 1; j < NI; j++) {
            tmem_ld<G>(ta + j * BN, t[j - 1]);
            tmem_ld<G>(tb + j * BN, t[j - 1] + G);
        }
        tc_wait_ld();
#pragma unroll
        for (int j = 1; j < NI; j++)
#pragma unroll
            for (int c = 0; c < 2 * G; c++) v[c] += t[j - 1][c];
    } else {
        tc_wait_ld();
    }
}

// Clears p.zero (a statistics buffer a later GEMM accumulates into), striding over nblk CTAs.
__device__ __forceinline__ void gemm_zero(const GemmParams &p, uint32_t blk, uint32_t nblk) {
    for (uint32_t i = blk * blockDim.x + threadIdx.x; i < p.zero_len; i += nblk * blockDim.x)
        p.zero[i] = 0.0f;
}

// The k-blocks of split z of `splits` for a k of kb_total blocks.
__device__ __forceinline__ void k_range(uint32_t kb_total, uint32_t z, uint32_t splits,
                                        uint32_t &kb0, uint32_t &nkb) {
    kb0 = z * kb_total / splits;
    nkb = (z + 1) * kb_total / splits - kb0;
}

// The shared::cluster address of local shared address `a` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}

// A barrier across the CTAs of a thread-block cluster (every thread of every CTA) in two halves:
// arrive (release) early, wait (acquire) when needed.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Four floats into shared memory of another CTA of the cluster (addr, remote_bar: its
// shared::cluster addresses), asynchronously: the 16 bytes count towards the transaction bytes of
// that CTA's mbarrier remote_bar.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float a, float b, float c, float d,
                                            uint32_t remote_bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
        "f"(a), "f"(b), "f"(c), "f"(d), "r"(remote_bar)
        : "memory");
}

// Cluster split-K set-up (every thread, after gemm_setup): the receive barrier armed for the bytes
// the peers will send, its initialisation released to the cluster. The matching cluster_wait comes
// before this CTA's first remote store, so every peer's barrier is armed by then.
template <int BN, int STAGES, int CS>
__device__ __forceinline__ void gemm_cluster_setup(const GemmSmemView<BN, STAGES> &sv) {
    if constexpr (CS > 1) {
        if (threadIdx.x == 0) {
            mbar_init(sv.recv_bar, 1);
            fence_barrier_init();
            mbar_arrive_expect_tx(sv.recv_bar, GemmShape<BN, STAGES>::template RECV_TX<CS>);
        }
        __syncthreads();
        cluster_arrive();
    }
}

// How a tile waits for its inputs (the activations, statistics and residuals a previous step
// writes): gate.producer() is called by the TMA thread after it has requested the first stages'
// weights and before it requests activations; gate.all() by every thread before the epilogue's
// loads. The single-GEMM kernel waits on programmatic dependent launch.
struct PdlGate {
    __device__ void producer() const { pdl_wait(); }
    __device__ void all() const {
        pdl_launch_dependents();
        pdl_wait();
    }
};

// One BM x BN output tile (split z of `splits`; `tile` numbers it for the split counters). Every
// thread of the CTA calls it. BM = 64 (an M = 64 MMA; its rows in lanes 0-15 of each warp's TMEM
// quadrant) serves single-CTA tiles only (no split, no cluster). `prefetched`: leading stages whose W half gemm_issue_w already
// issued. `gate`: how the tile waits for its inputs (PdlGate, or the persistent kernel's
// dependency counters).
//
// CS > 1: the CTA is rank z of a cluster of CS CTAs that split K for the same tile. After their
// MMAs the CTAs reduce-scatter the f32 partials through distributed shared memory: CTA c owns
// columns [Go c, Go (c + 1)) of each 32-column half of every 64-column chunk (so RoPE pairs and
// GeGLU input / gate pairs stay together), receives the other CTAs' partials of them into its own
// (now idle) stage memory, sums them in rank order (deterministic) and runs the epilogue on them.
template <int BN, int STAGES, uint32_t EPI, int CS = 1, class Gate = PdlGate, int BM = GEMM_BM>
__device__ __forceinline__ void gemm_tile(const GemmParams &p,
                                          const GemmSmemView<BN, STAGES, BM> &sv,
                                          uint32_t tmem, GemmRun &run, uint32_t tile_n,
                                          uint32_t tile_m, uint32_t z, uint32_t splits,
                                          uint32_t tile, uint32_t prefetched, const Gate &gate) {
    using S = GemmShape<BN, STAGES, BM>;
    constexpr int CH = S::CH, NCH = S::NCH, HALF = CH / 2;
    constexpr int GT = CH / (4 * CS);  // columns per thread per half-chunk group
    constexpr int GO = 2 * GT;         // columns a cluster rank owns per half-chunk group
    static_assert(CS == 1 || CH == 64, "cluster split-K needs 64-column chunks");
    static_assert(CS == 1 || BM == GEMM_BM, "cluster split-K runs 128-row tiles");
    static_assert(GT >= 4, "at least 4 columns per thread group");
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = tile_n * BN, m0 = tile_m * BM;
    const uint32_t rank = CS > 1 ? z : 0;
    uint32_t kb0, nkb;
    k_range(p.k / GEMM_BK, z, splits, kb0, nkb);

    // Column sums and biases are weights: fetch them before waiting for the previous kernel.
    // (threads 64 and up: warps 0 and 1 hold the TMA producer and an MMA issuer)
    for (uint32_t j = threadIdx.x - 64; threadIdx.x >= 64 && j < (uint32_t)BN; j += GEMM_THREADS - 64) {
        if constexpr ((EPI & JC_EPI_LN) != 0) sv.cs_s[j] = __ldg(p.colsum + n0 + j);
        if constexpr ((EPI & JC_EPI_BIAS) != 0) sv.bs_s[j] = __ldg(p.bias + n0 + j);
    }

    const uint32_t nst = gemm_stages(nkb);
    const uint32_t pre = nst < (uint32_t)STAGES ? nst : (uint32_t)STAGES;
    // Phase stamps (profiling runs only): thread 0 (the producer) and thread 32 (the first issuer).
    uint64_t *rec = (threadIdx.x & ~32u) == 0 ? prof_record(p.prof, p.prof_cap) : nullptr;
    bool ok = true;
    if (warp == 0 && lane == 0) {
        // TMA producer: weights of the first stages first (they do not depend on the previous
        // kernel), then the activations.
        ok = gemm_issue_w<BN, STAGES, BM>(p, sv, run.it, n0, kb0, prefetched < pre ? prefetched : pre,
                                          pre);
        gate.producer();
        prof_stamp(rec, 1);
        for (uint32_t i = 0; ok && i < pre; i++) gemm_issue_a<BN, STAGES, BM>(p, sv, run.it, m0, kb0, i);
    }

    // Epilogue geometry: warp w owns the tile rows of TMEM lanes 32(w%4)..+31 (rows 32(w%4)..+31
    // of a 128-row tile; rows 16(w%4)..+15 of a 64-row one, in its first 16 lanes) and half w/4 of
    // the columns it handles.
    const uint32_t quarter = warp & 3, half = warp >> 2;
    const bool lane_ok = lane < (uint32_t)S::RPW;
    const uint32_t row = quarter * S::RPW + (lane & (S::RPW - 1));
    const uint32_t r = m0 + row;
    const bool valid = lane_ok && r < p.m;
    const uint32_t pair0 = GO * rank + GT * half;  // first column of this thread's groups
    gate.all();

    // Everything the epilogue reads from the previous step, requested by every thread (the MMA
    // issuers included) before the main loop so its latency hides under the MMAs.
    float2 st_in = make_float2(0.f, 0.f);
    if constexpr ((EPI & JC_EPI_LN) != 0) {
        if (valid) st_in = *reinterpret_cast<const float2 *>(p.stats_in + 2 * (size_t)r);
    }
    constexpr int RES_W = (EPI & JC_EPI_RES) ? NCH * GT : 1;
    uint32_t resw[RES_W];
    if constexpr ((EPI & JC_EPI_RES) != 0) {
        if (valid) {
            const __half *src = p.res + (size_t)r * p.n + n0;
#pragma unroll
            for (int ci = 0; ci < NCH; ci++) {
                load_halves<GT>(src + ci * CH + pair0, resw + ci * GT);
                load_halves<GT>(src + ci * CH + HALF + pair0, resw + ci * GT + GT / 2);
            }
        }
    }
    // RoPE angles depend only on the position inside the head: one set serves every chunk.
    constexpr int ROPE_V = (EPI & JC_EPI_ROPE) ? GT / 2 : 1;
    float4 ropev[ROPE_V];
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        if (valid) {
            // Pair-group-major table: consecutive rows (the lanes of a warp) are consecutive
            // float4s, so each load instruction reads one contiguous 512-byte run.
            // Row r's position: r, or its offset in its request when requests are packed.
            const uint32_t pos = p.seg ? r - p.seg[r].x : r;
            const float4 *t4 = reinterpret_cast<const float4 *>(p.rope) + (size_t)(pair0 / 2) * p.rope_stride + pos;
#pragma unroll
            for (int i = 0; i < GT / 2; i++) ropev[i] = __ldg(t4 + (size_t)i * p.rope_stride);
        }
    }

    if (warp == 0 && lane == 0) {
        for (uint32_t i = pre; ok && i < nst; i++) {
            ok = gemm_issue_w<BN, STAGES, BM>(p, sv, run.it, n0, kb0, i, i + 1);
            if (ok) gemm_issue_a<BN, STAGES, BM>(p, sv, run.it, m0, kb0, i);
        }
    } else if (warp >= 1 && warp <= (uint32_t)S::NI && lane == 0) {
        // MMA issuer j = warp - 1: of each stage's 4 x kbs MMAs (BM x BN x 16 each), those whose
        // index is j modulo NI, into accumulator j.
        constexpr uint32_t idesc = umma_idesc_f16(BM, BN);
        const uint32_t j = warp - 1, acc = tmem + j * BN;
        bool started = false;
        for (uint32_t i = 0; i < nst; i++) {
            const uint32_t g = run.it + i, s = g % STAGES, round = g / STAGES;
            if (!mbar_wait(&sv.full[s], round & 1, JC_DEV_TIMEOUT_FULL)) break;
            if (i == 0 && j == 0) prof_stamp(rec, 2);
            tc_fence_after();
            const uint32_t kbs = nkb - i * GEMM_KPS < (uint32_t)GEMM_KPS ? nkb - i * GEMM_KPS : GEMM_KPS;
            uint8_t *st = sv.stages + s * S::STAGE_BYTES;
#pragma unroll
            for (uint32_t q = j; q < 4 * GEMM_KPS; q += S::NI) {
                const uint32_t kb = q / 4, kk = q % 4;
                if (kb < kbs) {
                    const uint64_t ad = umma_desc_sw128(smem_u32(st + kb * S::A_KB));
                    const uint64_t bd = umma_desc_sw128(smem_u32(st + S::A_BYTES + kb * S::W_KB));
                    // +32 bytes (2 in descriptor units) per 16-element K step inside a 128B row.
                    tc_mma_f16(acc, ad + 2 * kk, bd + 2 * kk, idesc, started);
                    started = true;
                }
            }
            tc_commit(&sv.empty[s]);
        }
        tc_commit(sv.done);
    }
    __syncwarp();

    const bool mma_ok =
        __syncthreads_and(mbar_wait_sleep(sv.done, run.tiles & 1, JC_DEV_TIMEOUT_MMA)) != 0;
    if (threadIdx.x == 0) prof_stamp(rec, 3);
    tc_fence_after();
    float mean = 0.f, rstd = 0.f;
    if constexpr ((EPI & JC_EPI_LN) != 0) {
        mean = st_in.x / (float)p.k;
        const float var = st_in.y / (float)p.k - mean * mean;
        rstd = rsqrtf(fmaxf(var, 0.0f) + p.eps);
    }
    const uint32_t lane_base = tmem + ((quarter * 32) << 16);
    bool run_epilogue = mma_ok;
    constexpr int RS = S::template RECV_STRIDE<CS>;
    const float *recv = sv.recv;

    if constexpr (CS > 1) {
        // Reduce-scatter through distributed shared memory: each CTA sends every peer the
        // partials of the columns that peer owns (its own receive buffer, so no peer's operands
        // are overwritten), completing on the peer's receive barrier, then waits on its own.
        cluster_wait();  // every peer's receive barrier is armed
        if (mma_ok) {
            const uint32_t recv_s = smem_u32(sv.recv), bar_s = smem_u32(sv.recv_bar);
#pragma unroll
            for (int ci = 0; ci < NCH; ci++)
#pragma unroll
                for (uint32_t o = 0; o < (uint32_t)CS; o++) {
                    if (o == rank) continue;
                    float t[2 * GT];
                    acc_ld2<GT, S::NI, BN>(lane_base + ci * CH + GO * o + GT * half,
                                           lane_base + ci * CH + HALF + GO * o + GT * half, t);
                    const uint32_t dst = map_to_rank(recv_s, o) +
                                         (uint32_t)((((rank * NCH + ci) * 128 + row) * RS + GT * half) * 4);
                    const uint32_t rbar = map_to_rank(bar_s, o);
#pragma unroll
                    for (int j = 0; j < GT; j += 4) {
                        st_async_v4(dst + j * 4, t[j], t[j + 1], t[j + 2], t[j + 3], rbar);
                        st_async_v4(dst + (GO + j) * 4, t[GT + j], t[GT + j + 1], t[GT + j + 2],
                                    t[GT + j + 3], rbar);
                    }
                }
        }
        // Every peer sends whatever happened to this CTA's own MMAs, so the wait always ends (or
        // gives up, bounded) before the CTA may leave with writes into its memory in flight.
        const bool got = mbar_wait_sleep(sv.recv_bar, 0, JC_DEV_TIMEOUT_SPLIT);
        run_epilogue = __syncthreads_and(mma_ok && got) != 0;
        // This CTA has sent and received everything; the kernel's last wait (gemm_cluster_exit)
        // keeps every CTA of the cluster resident until all have.
        cluster_arrive();
    } else if (splits > 1 && mma_ok) {
        float *mine = p.ws + ((size_t)tile * splits + z) * BN * BM;
#pragma unroll
        for (int ci = 0; ci < NCH; ci++) {
            float v[2 * GT];
            acc_ld2<GT, S::NI, BN>(lane_base + ci * CH + pair0, lane_base + ci * CH + HALF + pair0, v);
            if (lane_ok) {
#pragma unroll
                for (int j = 0; j < GT; j++) {
                    mine[(size_t)(ci * CH + pair0 + j) * BM + row] = v[j];
                    mine[(size_t)(ci * CH + HALF + pair0 + j) * BM + row] = v[GT + j];
                }
            }
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t old = atomicAdd(&p.counters[tile], 1u);
            const bool last = old == splits - 1;
            if (last) p.counters[tile] = 0;
            *sv.last_flag = last ? 1u : 0u;
        }
        __syncthreads();
        run_epilogue = *sv.last_flag != 0;
        __threadfence();
    }

    // The output tile is staged in the stage memory, free now that every MMA has completed, in
    // boxes of BW columns, then written by TMA stores (p.map_c) or by every thread with 16-byte
    // stores of whole 128-byte (64-byte) row segments.
    constexpr int W_OUT = (EPI & JC_EPI_GEGLU) ? BN / 2 : BN;
    constexpr int BW = W_OUT < 64 ? W_OUT : 64;
    constexpr bool CAN_STAGE = CS == 1 && (BW == 32 || BW == 64) && GT % 8 == 0;
    uint8_t *stage = CAN_STAGE ? sv.stages : nullptr;
    if (run_epilogue) {
        float s = 0.f, q = 0.f;
#pragma unroll
        for (int ci = 0; ci < NCH; ci++) {
            float v[2 * GT];
            const uint32_t ca = ci * CH + pair0, cb = ca + HALF;
            if constexpr (CS > 1) {
                // Sum the ranks' partials in rank order: this CTA's own from TMEM, the others
                // from its stage memory.
#pragma unroll
                for (int j = 0; j < 2 * GT; j++) v[j] = 0.0f;
#pragma unroll
                for (uint32_t zz = 0; zz < (uint32_t)CS; zz++) {
                    if (zz == rank) {
                        float t[2 * GT];
                        acc_ld2<GT, S::NI, BN>(lane_base + ca, lane_base + cb, t);
#pragma unroll
                        for (int j = 0; j < 2 * GT; j++) v[j] += t[j];
                    } else {
                        const float *src = recv + ((size_t)(zz * NCH + ci) * 128 + row) * RS + GT * half;
#pragma unroll
                        for (int j = 0; j < GT; j += 4) {
                            const float4 a4 = *reinterpret_cast<const float4 *>(src + j);
                            const float4 b4 = *reinterpret_cast<const float4 *>(src + GO + j);
                            v[j] += a4.x; v[j + 1] += a4.y; v[j + 2] += a4.z; v[j + 3] += a4.w;
                            v[GT + j] += b4.x; v[GT + j + 1] += b4.y; v[GT + j + 2] += b4.z;
                            v[GT + j + 3] += b4.w;
                        }
                    }
                }
            } else if (splits == 1) {
                acc_ld2<GT, S::NI, BN>(lane_base + ca, lane_base + cb, v);
            } else {
#pragma unroll
                for (int j = 0; j < 2 * GT; j++) v[j] = 0.0f;
                for (uint32_t zz = 0; zz < splits; zz++) {
                    if (zz == z) {
                        float t[2 * GT];
                        acc_ld2<GT, S::NI, BN>(lane_base + ca, lane_base + cb, t);
#pragma unroll
                        for (int j = 0; j < 2 * GT; j++) v[j] += t[j];
                    } else {
                        const float *part = p.ws + ((size_t)tile * splits + zz) * BN * BM;
#pragma unroll
                        for (int j = 0; j < GT; j++) {
                            v[j] += __ldcg(part + (size_t)(ca + j) * BM + row);
                            v[GT + j] += __ldcg(part + (size_t)(cb + j) * BM + row);
                        }
                    }
                }
            }
            gemm_epilogue_part<GT, HALF, EPI, BW, BM>(p, v, r, row, stage, valid, n0, n0 + ci * CH, pair0, mean, rstd,
                                              sv.cs_s, sv.bs_s, resw + ((EPI & JC_EPI_RES) ? ci * GT : 0),
                                              ropev, s, q);
        }
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            // The two halves of a row meet in shared memory; one atomic pair per row per CTA.
            if (half && lane_ok) sv.row_part[row] = make_float2(s, q);
            __syncthreads();
            if (!half && valid) {
                const float2 o = sv.row_part[row];
                red_add_f32x2(p.stats_out + 2 * (size_t)r, s + o.x, q + o.y);
            }
        }
        if (stage && p.map_c) {
            // Every thread's staging writes are visible to the TMA (async proxy) before one
            // thread stores the boxes (rows past m are not written) and waits until they have
            // been read out of shared memory.
            fence_proxy_async();
            __syncthreads();
            if (threadIdx.x == 0) {
                const int32_t out0 = (int32_t)((EPI & JC_EPI_GEGLU) ? n0 / 2 : n0);
#pragma unroll
                for (int b = 0; b < W_OUT / BW; b++)
                    tma_store_2d(p.map_c, stage + b * BM * BW * 2, out0 + b * BW, (int32_t)m0);
                bulk_commit();
                bulk_wait_read();
            }
        } else if (stage) {
            // Every thread copies 16-byte chunks out of the staged tile, consecutive threads
            // taking consecutive chunks of a row (rows past m are not written); the stores need
            // no wait.
            __syncthreads();
            constexpr uint32_t CPR = W_OUT / 8, CPB = BW / 8;  // 16-byte chunks a row, a box row
            const uint32_t ld = (EPI & JC_EPI_GEGLU) ? p.n / 2 : p.n;
            __half *out = p.c + ((EPI & JC_EPI_GEGLU) ? n0 / 2 : n0);
#pragma unroll 4
            for (uint32_t idx = threadIdx.x; idx < (uint32_t)BM * CPR; idx += GEMM_THREADS) {
                const uint32_t rr = idx / CPR, ch = idx % CPR, b = ch / CPB, c = ch % CPB;
                const uint32_t sw = BW == 64 ? (rr & 7) : ((rr >> 1) & 3);
                if (m0 + rr < p.m)
                    *reinterpret_cast<uint4 *>(out + (size_t)(m0 + rr) * ld + ch * 8) =
                        *reinterpret_cast<const uint4 *>(stage + b * BM * BW * 2 + rr * BW * 2 + ((c ^ sw) << 4));
            }
        }
    }
    // Every TMEM read and shared-memory use of this tile is done before the next one starts.
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) prof_stamp(rec, 4);
    run.it += nst;
    run.tiles += 1;
}

// The single-GEMM kernel: its tensor maps travel as kernel parameters.
struct GemmKernelParams {
    CUtensorMap map_a;
    CUtensorMap map_w;
    CUtensorMap map_c;  // valid when p.store_tma
    GemmParams p;
};

template <int BN, int STAGES, uint32_t EPI, int CS, int BM = GEMM_BM>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ GemmKernelParams kp) {
    dev_err_bind(kp.p.err);
    uint64_t *rec = threadIdx.x == 0 ? prof_record(kp.p.prof, kp.p.prof_cap) : nullptr;
    prof_open(rec);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    GemmParams p = kp.p;
    p.map_a = &kp.map_a;
    p.map_w = &kp.map_w;
    p.map_c = p.store_tma ? &kp.map_c : nullptr;
    const GemmSmemView<BN, STAGES, BM> sv(base);
    if (threadIdx.x == 32) {
        tma_prefetch_desc(p.map_a);
        tma_prefetch_desc(p.map_w);
    }
    const uint32_t tmem = gemm_setup<BN, STAGES, BM>(sv);
    if constexpr (CS > 1) gemm_cluster_setup<BN, STAGES, CS>(sv);
    GemmRun run;
    gemm_tile<BN, STAGES, EPI, CS, PdlGate, BM>(p, sv, tmem, run, blockIdx.x, blockIdx.y, blockIdx.z,
                                                gridDim.z, blockIdx.y * gridDim.x + blockIdx.x, 0,
                                                PdlGate{});
    gemm_zero(p, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
              gridDim.x * gridDim.y * gridDim.z);
    if constexpr (CS > 1) cluster_wait();  // no CTA leaves while a peer may still write into it
    gemm_teardown<BN, STAGES>(tmem);
    prof_stamp(rec, 5);
}

}  // namespace jc
