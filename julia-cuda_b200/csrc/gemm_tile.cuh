// One GEMM output tile as a device function (the body of both the single-GEMM kernel and of the
// persistent kernel's GEMM phases), its set-up / tear-down, and the single-GEMM kernel.
#pragma once
#include "gemm.cuh"

namespace jc {

// Where a CTA's GEMM pipeline lives in shared memory: STAGES stages, then the barriers, the TMEM
// base slot, a flag, per-row partial statistics and the tile's column sums / biases.
template <int BN, int STAGES>
struct GemmSmemView {
    using S = GemmShape<BN, STAGES>;
    uint8_t *stages;
    uint64_t *full, *empty, *done;
    uint32_t *tmem_slot, *last_flag;
    float2 *row_part;
    float *cs_s, *bs_s;
    __device__ explicit GemmSmemView(uint8_t *base) {
        stages = base;
        uint8_t *tail = base + STAGES * S::STAGE_BYTES;
        full = reinterpret_cast<uint64_t *>(tail);
        empty = full + STAGES;
        done = empty + STAGES;
        tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
        last_flag = tmem_slot + 1;
        row_part = reinterpret_cast<float2 *>(tail + 256);
        cs_s = reinterpret_cast<float *>(tail + 256 + 1024);
        bs_s = cs_s + BN;
    }
};

// A CTA's pipeline position across tiles (every thread keeps the same copy): k-blocks issued so
// far (stage = it % STAGES, ring round = it / STAGES) and tiles finished (the accumulator
// barrier's parity).
struct GemmRun {
    uint32_t it = 0;
    uint32_t tiles = 0;
};

// Barrier initialisation and the TMEM accumulator; every thread calls it, returns the TMEM base.
template <int BN, int STAGES>
__device__ __forceinline__ uint32_t gemm_setup(const GemmSmemView<BN, STAGES> &sv) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&sv.full[s], 1);
            mbar_init(&sv.empty[s], 1);
        }
        mbar_init(sv.done, 1);
        fence_barrier_init();
    }
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

// Producer thread only: the W half of the first `count` stages of a tile whose pipeline starts at
// run.it (expect_tx covers A and W; the A halves follow once the activations are ready).
template <int BN, int STAGES>
__device__ __forceinline__ bool gemm_issue_w(const GemmParams &p, const GemmSmemView<BN, STAGES> &sv,
                                             uint32_t it, uint32_t n0, uint32_t kb0,
                                             uint32_t first, uint32_t count) {
    using S = GemmShape<BN, STAGES>;
    for (uint32_t i = first; i < count; i++) {
        const uint32_t g = it + i, s = g % STAGES, round = g / STAGES;
        if (round > 0 && !mbar_wait(&sv.empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY))
            return false;
        uint8_t *st = sv.stages + s * S::STAGE_BYTES;
        mbar_arrive_expect_tx(&sv.full[s], S::STAGE_BYTES);
        tma_load_2d(st + S::A_BYTES, p.map_w, &sv.full[s], (int32_t)((kb0 + i) * GEMM_BK),
                    (int32_t)n0);
    }
    return true;
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

// One 128 x BN output tile (split z of `splits`; `tile` numbers it for the split counters). Every
// thread of the CTA calls it. `prefetched`: leading stages whose W half gemm_issue_w already
// issued. `standalone`: the single-GEMM kernel (programmatic dependent launch waits here); in the
// persistent kernel a grid barrier has already ordered the inputs.
template <int BN, int STAGES, uint32_t EPI>
__device__ __forceinline__ void gemm_tile(const GemmParams &p, const GemmSmemView<BN, STAGES> &sv,
                                          uint32_t tmem, GemmRun &run, uint32_t tile_n,
                                          uint32_t tile_m, uint32_t z, uint32_t splits,
                                          uint32_t tile, uint32_t prefetched, bool standalone) {
    using S = GemmShape<BN, STAGES>;
    constexpr int CH = S::CH, G = S::G, NCH = S::NCH;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = tile_n * BN, m0 = tile_m * GEMM_BM;
    uint32_t kb0, nkb;
    k_range(p.k / GEMM_BK, z, splits, kb0, nkb);

    // Column sums and biases are weights: fetch them before waiting for the previous kernel.
    if (threadIdx.x >= 64 && threadIdx.x < 64 + BN) {
        const uint32_t j = threadIdx.x - 64;
        if constexpr ((EPI & JC_EPI_LN) != 0) sv.cs_s[j] = __ldg(p.colsum + n0 + j);
        if constexpr ((EPI & JC_EPI_BIAS) != 0) sv.bs_s[j] = __ldg(p.bias + n0 + j);
    }

    if (warp == 0 && lane == 0) {
        // TMA producer: weights of the first stages first (they do not depend on the previous
        // kernel), then the activations.
        const uint32_t pre = nkb < (uint32_t)STAGES ? nkb : (uint32_t)STAGES;
        bool ok = gemm_issue_w<BN, STAGES>(p, sv, run.it, n0, kb0, prefetched < pre ? prefetched : pre, pre);
        if (standalone) pdl_wait();
        for (uint32_t i = 0; ok && i < pre; i++) {
            const uint32_t s = (run.it + i) % STAGES;
            tma_load_2d(sv.stages + s * S::STAGE_BYTES, p.map_a, &sv.full[s],
                        (int32_t)((kb0 + i) * GEMM_BK), (int32_t)m0);
        }
        for (uint32_t i = pre; ok && i < nkb; i++) {
            const uint32_t g = run.it + i, s = g % STAGES, round = g / STAGES;
            if (!mbar_wait(&sv.empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY)) break;
            uint8_t *st = sv.stages + s * S::STAGE_BYTES;
            mbar_arrive_expect_tx(&sv.full[s], S::STAGE_BYTES);
            tma_load_2d(st + S::A_BYTES, p.map_w, &sv.full[s], (int32_t)((kb0 + i) * GEMM_BK),
                        (int32_t)n0);
            tma_load_2d(st, p.map_a, &sv.full[s], (int32_t)((kb0 + i) * GEMM_BK), (int32_t)m0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: 4 x (128 x BN x 16) per 64-deep K block.
        constexpr uint32_t idesc = umma_idesc_f16(GEMM_BM, BN);
        for (uint32_t i = 0; i < nkb; i++) {
            const uint32_t g = run.it + i, s = g % STAGES, round = g / STAGES;
            if (!mbar_wait(&sv.full[s], round & 1, JC_DEV_TIMEOUT_FULL)) break;
            tc_fence_after();
            uint8_t *st = sv.stages + s * S::STAGE_BYTES;
            const uint64_t ad = umma_desc_sw128(smem_u32(st));
            const uint64_t bd = umma_desc_sw128(smem_u32(st + S::A_BYTES));
#pragma unroll
            for (uint32_t kk = 0; kk < GEMM_BK / 16; kk++)
                // +32 bytes (2 in descriptor units) per 16-element K step inside the 128B row.
                tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0);
            tc_commit(&sv.empty[s]);
        }
        tc_commit(sv.done);
    }
    __syncwarp();

    // ---- epilogue: warp w owns rows 32(w%4)..+31 and column half w/4 of each chunk ----
    const uint32_t quarter = warp & 3, half = warp >> 2;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t r = m0 + row;
    const bool valid = r < p.m;
    if (standalone) {
        pdl_launch_dependents();
        pdl_wait();
    }

    // Everything the epilogue reads from the previous step, fetched while the MMAs run.
    float mean = 0.f, rstd = 0.f;
    if constexpr ((EPI & JC_EPI_LN) != 0) {
        if (valid) {
            const float2 st = *reinterpret_cast<const float2 *>(p.stats_in + 2 * (size_t)r);
            mean = st.x / (float)p.k;
            const float var = st.y / (float)p.k - mean * mean;
            rstd = rsqrtf(fmaxf(var, 0.0f) + p.eps);
        }
    }
    constexpr int RES_V = (EPI & JC_EPI_RES) ? NCH * 2 * G / 8 : 1;
    uint4 resv[RES_V];
    if constexpr ((EPI & JC_EPI_RES) != 0) {
        if (valid) {
            const uint4 *src = reinterpret_cast<const uint4 *>(p.res + (size_t)r * p.n + n0);
#pragma unroll
            for (int ci = 0; ci < NCH; ci++)
#pragma unroll
                for (int j = 0; j < G / 8; j++) {
                    resv[ci * 2 * G / 8 + j] = src[(ci * CH + G * half) / 8 + j];
                    resv[ci * 2 * G / 8 + G / 8 + j] = src[(ci * CH + CH / 2 + G * half) / 8 + j];
                }
        }
    }
    constexpr int ROPE_V = (EPI & JC_EPI_ROPE) ? NCH * 8 : 1;
    float4 ropev[ROPE_V];
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        if (valid) {
            const float4 *t4 = reinterpret_cast<const float4 *>(p.rope + (size_t)r * 64 + 32 * half);
#pragma unroll
            for (int ci = 0; ci < NCH; ci++)
#pragma unroll
                for (int i = 0; i < 8; i++) ropev[ci * 8 + i] = __ldg(t4 + i);
        }
    }

    const bool mma_ok =
        __syncthreads_and(mbar_wait_sleep(sv.done, run.tiles & 1, JC_DEV_TIMEOUT_MMA)) != 0;
    tc_fence_after();
    const uint32_t lane_base = tmem + ((quarter * 32) << 16);
    bool run_epilogue = mma_ok;

    if (splits > 1 && mma_ok) {
        float *mine = p.ws + ((size_t)tile * splits + z) * BN * GEMM_BM;
#pragma unroll 1
        for (int cb = 0; cb < BN; cb += CH) {
            float v[2 * G];
            tmem_ld<G>(lane_base + cb + G * half, v);
            tmem_ld<G>(lane_base + cb + CH / 2 + G * half, v + G);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < G; j++) {
                mine[(size_t)(cb + G * half + j) * GEMM_BM + row] = v[j];
                mine[(size_t)(cb + CH / 2 + G * half + j) * GEMM_BM + row] = v[G + j];
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

    if (run_epilogue) {
        float s = 0.f, q = 0.f;
#pragma unroll
        for (int ci = 0; ci < NCH; ci++) {
            float v[2 * G];
            const uint32_t la = ci * CH + G * half, lb = la + CH / 2;
            if (splits == 1) {
                tmem_ld<G>(lane_base + la, v);
                tmem_ld<G>(lane_base + lb, v + G);
                tc_wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < 2 * G; j++) v[j] = 0.0f;
                for (uint32_t zz = 0; zz < splits; zz++) {
                    if (zz == z) {
                        float t[2 * G];
                        tmem_ld<G>(lane_base + la, t);
                        tmem_ld<G>(lane_base + lb, t + G);
                        tc_wait_ld();
#pragma unroll
                        for (int j = 0; j < 2 * G; j++) v[j] += t[j];
                    } else {
                        const float *part = p.ws + ((size_t)tile * splits + zz) * BN * GEMM_BM;
#pragma unroll
                        for (int j = 0; j < G; j++) {
                            v[j] += __ldcg(part + (size_t)(la + j) * GEMM_BM + row);
                            v[G + j] += __ldcg(part + (size_t)(lb + j) * GEMM_BM + row);
                        }
                    }
                }
            }
            gemm_epilogue_part<CH, EPI>(p, v, r, valid, n0, la, half, mean, rstd, sv.cs_s, sv.bs_s,
                                        resv + ((EPI & JC_EPI_RES) ? ci * 2 * G / 8 : 0),
                                        ropev + ((EPI & JC_EPI_ROPE) ? ci * 8 : 0), s, q);
        }
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            // The two halves of a row meet in shared memory; one atomic pair per row per tile.
            if (half) sv.row_part[row] = make_float2(s, q);
            __syncthreads();
            if (!half && valid) {
                const float2 o = sv.row_part[row];
                atomicAdd(p.stats_out + 2 * (size_t)r, s + o.x);
                atomicAdd(p.stats_out + 2 * (size_t)r + 1, q + o.y);
            }
        }
    }
    // Every TMEM read and shared-memory use of this tile is done before the next one starts.
    tc_fence_before();
    __syncthreads();
    run.it += nkb;
    run.tiles += 1;
}

// The single-GEMM kernel: its tensor maps travel as kernel parameters.
struct GemmKernelParams {
    CUtensorMap map_a;
    CUtensorMap map_w;
    GemmParams p;
};

template <int BN, int STAGES, uint32_t EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ GemmKernelParams kp) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    GemmParams p = kp.p;
    p.map_a = &kp.map_a;
    p.map_w = &kp.map_w;
    const GemmSmemView<BN, STAGES> sv(base);
    if (threadIdx.x == 32) {
        tma_prefetch_desc(p.map_a);
        tma_prefetch_desc(p.map_w);
    }
    const uint32_t tmem = gemm_setup<BN, STAGES>(sv);
    GemmRun run;
    gemm_tile<BN, STAGES, EPI>(p, sv, tmem, run, blockIdx.x, blockIdx.y, blockIdx.z, gridDim.z,
                               blockIdx.y * gridDim.x + blockIdx.x, 0, true);
    gemm_zero(p, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
              gridDim.x * gridDim.y * gridDim.z);
    gemm_teardown<BN, STAGES>(tmem);
}

}  // namespace jc
