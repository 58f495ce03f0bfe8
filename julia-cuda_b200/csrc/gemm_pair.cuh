// The fused-epilogue GEMM on CTA pairs, for launches of many tiles (large packs of requests):
// a cluster of two CTAs on two SMs computes 256 x BN output tiles with tcgen05 MMAs of
// cta_group::2 (M = 256), and walks its tiles persistently as gemm_persist.cuh does.
//
// Why pairs: a single-SM 128 x 256 tile streams 128 activation rows and 256 weight rows per
// k-block for 128 x 256 outputs; the pair streams, per SM, its own 128 activation rows and half
// of the 256 weight rows (the MMA reads the other half from the peer's shared memory), so each SM
// ingests a third fewer operand bytes per output. At thousands of rows the single-SM kernel is
// bound by that stream, not by the tensor pipe. No TMA multicast is involved: every load reads
// global memory into the loading CTA's own shared memory.
//
//   - CTA rank r of the pair holds rows [m0 + 128 r, m0 + 128 r + 128) of the tile's activations
//     and weight rows [n0 + r BN / 2, n0 + (r + 1) BN / 2), each k-block as one 3-D TMA box, in
//     the same STAGES-deep ring at the same shared-memory offsets in both CTAs;
//   - both CTAs' loads complete on the leader's (rank 0) full barrier (the cta_group::2 form of
//     the TMA load may signal the peer's barrier); the leader's producer alone arms it with both
//     CTAs' bytes;
//   - lane 0 of the leader's warp 1 issues every MMA (M = 256, N = BN, K = 16): rank r's TMEM
//     receives rows 128 r .. 128 r + 127 of the tile, all BN columns, in one of two accumulator
//     buffers; each stage is released in both CTAs by one tcgen05.commit multicast to both empty
//     barriers, each finished tile by one commit multicast to both accumulator-full barriers;
//   - warps 4 and up of each CTA run the epilogue of its 128 rows (persist_tile_epilogue, as
//     gemm_persist.cuh) and report the buffer free on the leader's accumulator-empty barrier
//     (one arrival for each epilogue warp of both CTAs);
//   - warp 3 clears the statistics buffer a later GEMM adds into.
// TMEM is allocated and freed with cta_group::2 by warp 0 of both CTAs; a cluster barrier after
// the set-up (barriers initialised before any peer signals them) and one before the teardown
// (every MMA and every epilogue read done) bracket the tile loop. Every wait is bounded.
#pragma once
#include "gemm_persist.cuh"

namespace jc {

template <int BN, int STAGES_>
struct GemmPairShape {
    static constexpr int STAGES = STAGES_;
    static constexpr int A_KB = GEMM_BM * GEMM_BK * 2;   // this CTA's 128 rows of a k-block
    static constexpr int W_KB = (BN / 2) * GEMM_BK * 2;  // this CTA's half of the weight rows
    static constexpr int A_BYTES = GEMM_KPS * A_KB;
    static constexpr int STAGE_BYTES = A_BYTES + GEMM_KPS * W_KB;
    // stages | barriers (1 KB) | the epilogue warps' buffers
    static constexpr int EPI_OFF = STAGES * STAGE_BYTES + 1024;
    static constexpr int SMEM_BYTES = EPI_OFF + PERSIST_EPI_BYTES;
    static_assert(BN == 128 || BN == 256, "pair tiles are 128 or 256 columns wide");
    static_assert(2 * BN <= 512, "two accumulator buffers in TMEM");
    static_assert(STAGE_BYTES % 1024 == 0 && W_KB % 1024 == 0, "stages keep 1024-byte alignment");
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// 3-D tiled load into this CTA's shared memory, completing on the barrier at shared::cluster
// address `bar` (the pair leader's). No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the barrier at this shared-memory offset in both CTAs of the pair when every
// MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}

// Arrive on a barrier of another CTA of the cluster (shared::cluster address), releasing this
// thread's earlier accesses at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <int BN, int STAGES, uint32_t EPI>
__global__ void __launch_bounds__(PERSIST_GEMM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ GemmKernelParams kp) {
    dev_err_bind(kp.p.err);
    using S = GemmPairShape<BN, STAGES>;
    constexpr int PAIR_M = 2 * GEMM_BM;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    GemmParams p = kp.p;
    p.map_a = &kp.map_a;
    p.map_w = &kp.map_w;
    uint64_t *full = reinterpret_cast<uint64_t *>(base + STAGES * S::STAGE_BYTES);
    uint64_t *empty = full + STAGES, *acc_full = empty + STAGES, *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);   // the leader's producer; both CTAs' bytes
            mbar_init(&empty[s], 1);  // the leader's commit, multicast
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);   // the leader's commit, multicast
            mbar_init(&acc_empty[b], 8 * PERSIST_EPI_CG);  // lane 0 of every epilogue warp of both CTAs
        }
        fence_barrier_init();
    }
    if (threadIdx.x == 32) {
        tma_prefetch_desc(p.map_a);
        tma_prefetch_desc(p.map_w);
    }
    if (warp == 0) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    // Both CTAs' barriers are initialised (and TMEM allocated) before either signals the other.
    cluster_arrive();
    cluster_wait();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const uint32_t tiles_n = p.n / BN, tiles_m = (p.m + PAIR_M - 1) / PAIR_M;
    const uint32_t total = tiles_m * tiles_n, nst = gemm_stages(p.k / GEMM_BK);
    const uint32_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = map_to_rank(smem_u32(full), 0);
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < total; t += pairs) {
                const uint32_t m0 = (t / tiles_n) * PAIR_M + rank * GEMM_BM;
                const uint32_t n0 = (t % tiles_n) * BN + rank * (BN / 2);
                for (uint32_t st = 0; st < nst; st++, g++) {
                    const uint32_t s = g % STAGES, round = g / STAGES;
                    if (round > 0 && !mbar_wait(&empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *stage = base + s * S::STAGE_BYTES;
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * S::STAGE_BYTES);
                    tma_load_3d_pair(stage + S::A_BYTES, p.map_w, full0 + s * 8, 0, (int32_t)n0,
                                     (int32_t)(st * GEMM_KPS));
                    if (g == 0) {
                        pdl_wait();
                        pdl_launch_dependents();
                    }
                    tma_load_3d_pair(stage, p.map_a, full0 + s * 8, 0, (int32_t)m0, (int32_t)(st * GEMM_KPS));
                }
            }
            // Every stage's last release (the leader's commit, multicast to this CTA too) has
            // arrived before this CTA may leave.
            for (uint32_t j = 0; ok && j < (uint32_t)STAGES; j++, g++) {
                const uint32_t s = g % STAGES, round = g / STAGES;
                if (round > 0 && !mbar_wait(&empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY)) ok = false;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(PAIR_M, BN);
            const uint32_t kbs_total = p.k / GEMM_BK;
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t t = pair, i = 0; ok && t < total; t += pairs, i++) {
                const uint32_t buf = i & 1, acc = tmem + buf * BN;
                // Both CTAs' epilogues have read this buffer's previous tile (two tiles ago).
                if (i >= 2 && !mbar_wait(&acc_empty[buf], ((i - 2) >> 1) & 1, JC_DEV_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                bool started = false;
                for (uint32_t st = 0; st < nst; st++, g++) {
                    const uint32_t s = g % STAGES, round = g / STAGES;
                    if (!mbar_wait(&full[s], round & 1, JC_DEV_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kbs = kbs_total - st * GEMM_KPS < (uint32_t)GEMM_KPS ? kbs_total - st * GEMM_KPS : GEMM_KPS;
                    uint8_t *stage = base + s * S::STAGE_BYTES;
#pragma unroll
                    for (uint32_t qq = 0; qq < 4 * GEMM_KPS; qq++) {
                        const uint32_t kb = qq / 4, kk = qq % 4;
                        if (kb < kbs) {
                            const uint64_t ad = umma_desc_sw128(smem_u32(stage + kb * S::A_KB));
                            const uint64_t bd = umma_desc_sw128(smem_u32(stage + S::A_BYTES + kb * S::W_KB));
                            tc_mma_f16_pair(acc, ad + 2 * kk, bd + 2 * kk, idesc, started);
                            started = true;
                        }
                    }
                    tc_commit_pair(&empty[s]);
                }
                if (ok) tc_commit_pair(&acc_full[buf]);
            }
        }
    } else if (warp == 3) {
        pdl_wait();
        pdl_launch_dependents();
        // This warp alone clears the buffer, striding over every CTA's warp 3.
        for (uint32_t i = blockIdx.x * 32 + lane; i < p.zero_len; i += gridDim.x * 32) p.zero[i] = 0.0f;
    } else if (warp >= 4) {
        // Epilogue of this CTA's 128 rows of each tile.
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t quarter = warp & 3, grp = (warp - 4) >> 2;
        const uint32_t lane_base = tmem + ((quarter * 32) << 16);
        const uint32_t acc_empty0 = map_to_rank(smem_u32(acc_empty), 0);
        uint8_t *qbuf = base + S::EPI_OFF + quarter * PERSIST_EPI_QUARTER_BYTES;
        for (uint32_t t = pair, i = 0; t < total; t += pairs, i++) {
            const uint32_t buf = i & 1;
            const uint32_t m0 = (t / tiles_n) * PAIR_M + rank * GEMM_BM, n0 = (t % tiles_n) * BN;
            // The leader's MMAs of the tile after next may overwrite this buffer once every
            // epilogue warp of the pair has read its part.
            if (!persist_tile_epilogue<BN, 1, EPI>(p, lane_base + buf * BN, &acc_full[buf], (i >> 1) & 1, qbuf,
                                                   quarter, grp, lane, m0, n0, [&] {
                                                       if (rank == 0)
                                                           mbar_arrive(&acc_empty[buf]);
                                                       else
                                                           mbar_arrive_remote(acc_empty0 + buf * 8);
                                                   }))
                break;
        }
    }
    // Every MMA into either CTA's TMEM has completed and both epilogues have read it (or given
    // up) before the pair frees it.
    tc_fence_before();
    __syncthreads();
    cluster_arrive();
    cluster_wait();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

}  // namespace jc
