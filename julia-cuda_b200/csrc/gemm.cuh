// The encoder's fused-epilogue GEMM family on sm_100a tensor cores.
//
// c = epilogue(a . w^T): a [m, k] f16 row-major (activations), w [n, k] f16 row-major (nn.Linear
// weights), f32 accumulation in tensor memory. Replaces the reference's mma.sync family
// (kernels/src/gemm.rs:317-433 mainloop / split_reduce, kernels/src/main.rs:886-1147 gemm_tile
// and its 32 instances) with one tcgen05 design:
//
//   - a CTA computes a 128 x BN tile (BN = 32, 64 or 128) with 256 threads;
//   - warp 0 lane 0 streams 64-deep K blocks of A and W into a ring of STAGES 128B-swizzled
//     shared-memory stages with TMA (no multicast), each stage completing on an mbarrier;
//   - warp 1 lane 0 issues tcgen05.mma (M=128, N=BN, K=16, kind::f16) into a TMEM accumulator and
//     releases each stage with tcgen05.commit;
//   - meanwhile the other warps fetch everything the epilogue reads (column sums and biases into
//     shared memory, each row's LayerNorm statistics, residuals and RoPE angles into registers),
//     so no global round trip is left after the accumulator is ready;
//   - all eight warps run the epilogue: warp w reads TMEM lanes 32(w%4)..+31 (tile rows) and one
//     half of every 64-column chunk: columns [16h, 16h + 16) and [32 + 16h, 32 + 16h + 16) with
//     h = w / 4, so each thread holds both members of its RoPE pairs (i, i + 32) and both the GELU
//     inputs and the gates of its GeGLU outputs. No shuffles: q and k stay in natural (checkpoint)
//     order, and Wi's rows only need interleaving in blocks of 32 (prep_interleave_geglu), not the
//     reference's fragment-level permutations (src/prep.rs:67-101).
//
// Split-K (gridDim.z > 1): every split stores its f32 partial tile to `ws`, the last split of a
// tile to arrive (atomic counter, reset by it) sums all partials in split order, so the result
// does not depend on arrival order (the reference's scheme, kernels/src/gemm.rs:364-433), then
// runs the epilogue.
//
// Programmatic dependent launch: the weight tiles of the first stages (and the column sums and
// biases) are requested before griddepcontrol.wait, so they stream in while the previous kernel
// drains; activations, statistics and residuals are read only after it.
#pragma once
#include "common.cuh"

namespace jc {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 256;

struct GemmParams {
    CUtensorMap map_a;
    CUtensorMap map_w;
    __half *c;
    const __half *res;
    float *ws;
    uint32_t *counters;
    const float *stats_in;
    const float *colsum;
    float *stats_out;
    float *zero;
    const float *rope;
    const float *bias;
    uint32_t zero_len, m, n, k;
    float eps;
};

template <int BN, int STAGES_>
struct GemmShape {
    static constexpr int STAGES = STAGES_;
    static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
    static constexpr int B_BYTES = BN * GEMM_BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int CH = BN < 64 ? BN : 64;  // epilogue chunk
    static constexpr int G = CH / 4;              // columns per thread per half-chunk group
    static constexpr int NCH = BN / CH;           // chunks per tile
    static constexpr int PER = 2 * G * NCH;       // columns per thread
    // stages | barriers (256 B) | row partial sums (1 KB) | column sums and biases (2 x BN floats)
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + 1024 + 8 * BN;
    static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
};

// Stores G values (plus the residual, already in registers, and their statistics) at dst.
template <int G, uint32_t EPI>
__device__ __forceinline__ void store_group(const float *v, __half *dst, const uint4 *resv,
                                            float &s, float &q) {
#pragma unroll
    for (int j = 0; j < G / 8; j++) {
        float w[8];
#pragma unroll
        for (int e = 0; e < 8; e++) w[e] = v[8 * j + e];
        if constexpr ((EPI & JC_EPI_RES) != 0) {
            const uint4 rr = resv[j];
            const float2 a = unpack_half2(rr.x), b = unpack_half2(rr.y);
            const float2 cc = unpack_half2(rr.z), d = unpack_half2(rr.w);
            w[0] += a.x; w[1] += a.y; w[2] += b.x; w[3] += b.y;
            w[4] += cc.x; w[5] += cc.y; w[6] += d.x; w[7] += d.y;
        }
        uint4 o;
        o.x = pack_half2(w[0], w[1]);
        o.y = pack_half2(w[2], w[3]);
        o.z = pack_half2(w[4], w[5]);
        o.w = pack_half2(w[6], w[7]);
        reinterpret_cast<uint4 *>(dst)[j] = o;
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            // Statistics of the values as stored (f16), as the next LayerNorm sees them.
            const uint32_t pk[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = unpack_half2(pk[e]);
                s += f.x + f.y;
                q = fmaf(f.x, f.x, q);
                q = fmaf(f.y, f.y, q);
            }
        }
    }
}

// The epilogue of one thread's share of chunk `ci`: v[0, G) are tile columns la.., v[G, 2G) tile
// columns la + CH/2.. (la = ci * CH + G * half). cs / bs: the tile's column sums / biases in
// shared memory. For RoPE / GeGLU chunks (CH = 64) the pair index of v[j] / v[G + j] is 16h + j.
template <int CH, uint32_t EPI>
__device__ __forceinline__ void gemm_epilogue_part(const GemmParams &p, float *v, uint32_t r,
                                                   bool valid, uint32_t n0, uint32_t la,
                                                   uint32_t half, float mean, float rstd,
                                                   const float *cs, const float *bs,
                                                   const uint4 *resv, const float4 *ropev,
                                                   float &s, float &q) {
    constexpr int G = CH / 4;
    const uint32_t lb = la + CH / 2;
    if constexpr ((EPI & JC_EPI_LN) != 0) {
#pragma unroll
        for (int j = 0; j < G; j++) {
            v[j] = rstd * (v[j] - mean * cs[la + j]);
            v[G + j] = rstd * (v[G + j] - mean * cs[lb + j]);
        }
    }
    if constexpr ((EPI & JC_EPI_BIAS) != 0) {
#pragma unroll
        for (int j = 0; j < G; j++) {
            v[j] += bs[la + j];
            v[G + j] += bs[lb + j];
        }
    }
    if constexpr ((EPI & JC_EPI_RELU) != 0) {
#pragma unroll
        for (int j = 0; j < 2 * G; j++) v[j] = fmaxf(v[j], 0.0f);
    }
    if constexpr ((EPI & JC_EPI_GELU) != 0) {
#pragma unroll
        for (int j = 0; j < 2 * G; j++) v[j] = gelu_as(v[j]);
    }
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        static_assert(CH == 64, "RoPE needs whole 64-column heads");
        // q and k are the first two thirds of a qkv row; the chunk is exactly one head.
        if (valid && n0 + la < 2 * (p.n / 3)) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 t = ropev[i];  // (cos, sin) of pairs 16h + 2i and 16h + 2i + 1
                float x1 = v[2 * i], x2 = v[2 * i + 16];
                v[2 * i] = x1 * t.x - x2 * t.y;
                v[2 * i + 16] = x2 * t.x + x1 * t.y;
                x1 = v[2 * i + 1];
                x2 = v[2 * i + 17];
                v[2 * i + 1] = x1 * t.z - x2 * t.w;
                v[2 * i + 17] = x2 * t.z + x1 * t.w;
            }
        }
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
        static_assert(CH == 64, "GeGLU needs 32 input and 32 gate columns per chunk");
        if (valid) {
            // Packed columns [c0, c0 + 32) are GELU inputs of output columns [c0/2, c0/2 + 32),
            // [c0 + 32, c0 + 64) their gates; this thread has inputs / gates 16h .. 16h + 15.
            const uint32_t c0 = n0 + la - 16 * half;
            uint4 *dst = reinterpret_cast<uint4 *>(p.c + (size_t)r * (p.n / 2) + c0 / 2 + 16 * half);
#pragma unroll
            for (int j = 0; j < 2; j++) {
                uint4 o;
                o.x = pack_half2(gelu_as(v[8 * j + 0]) * v[8 * j + 16],
                                 gelu_as(v[8 * j + 1]) * v[8 * j + 17]);
                o.y = pack_half2(gelu_as(v[8 * j + 2]) * v[8 * j + 18],
                                 gelu_as(v[8 * j + 3]) * v[8 * j + 19]);
                o.z = pack_half2(gelu_as(v[8 * j + 4]) * v[8 * j + 20],
                                 gelu_as(v[8 * j + 5]) * v[8 * j + 21]);
                o.w = pack_half2(gelu_as(v[8 * j + 6]) * v[8 * j + 22],
                                 gelu_as(v[8 * j + 7]) * v[8 * j + 23]);
                dst[j] = o;
            }
        }
    } else {
        if (valid) {
            __half *row = p.c + (size_t)r * p.n + n0;
            store_group<G, EPI>(v, row + la, resv, s, q);
            store_group<G, EPI>(v + G, row + lb, resv + G / 8, s, q);
        }
    }
}

template <int BN, int STAGES, uint32_t EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    using S = GemmShape<BN, STAGES>;
    constexpr int CH = S::CH, G = S::G, NCH = S::NCH;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint8_t *tail = smem + STAGES * S::STAGE_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(tail);
    uint64_t *empty = full + STAGES;
    uint64_t *done = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    uint32_t *last_flag = tmem_slot + 1;
    float2 *row_part = reinterpret_cast<float2 *>(tail + 256);
    float *cs_s = reinterpret_cast<float *>(tail + 256 + 1024);
    float *bs_s = cs_s + BN;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * GEMM_BM;
    const uint32_t z = blockIdx.z, splits = gridDim.z;
    const uint32_t kb_total = p.k / GEMM_BK;
    const uint32_t kb0 = z * kb_total / splits, kb1 = (z + 1) * kb_total / splits;
    const uint32_t nkb = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (threadIdx.x == 32) {
        tma_prefetch_desc(&p.map_a);
        tma_prefetch_desc(&p.map_w);
    }
    // Column sums and biases are weights: fetch them before waiting for the previous kernel.
    if (threadIdx.x >= 64 && threadIdx.x < 64 + BN) {
        const uint32_t j = threadIdx.x - 64;
        if constexpr ((EPI & JC_EPI_LN) != 0) cs_s[j] = __ldg(p.colsum + n0 + j);
        if constexpr ((EPI & JC_EPI_BIAS) != 0) bs_s[j] = __ldg(p.bias + n0 + j);
    }
    if (warp == 0) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer. The weight tiles of the first stages do not depend on the previous
        // kernel: request them before waiting for it.
        const uint32_t pre = nkb < (uint32_t)STAGES ? nkb : (uint32_t)STAGES;
        for (uint32_t i = 0; i < pre; i++) {
            uint8_t *st = smem + i * S::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[i], S::STAGE_BYTES);
            tma_load_2d(st + S::A_BYTES, &p.map_w, &full[i], (int32_t)((kb0 + i) * GEMM_BK),
                        (int32_t)n0);
        }
        pdl_wait();
        for (uint32_t i = 0; i < pre; i++)
            tma_load_2d(smem + i * S::STAGE_BYTES, &p.map_a, &full[i],
                        (int32_t)((kb0 + i) * GEMM_BK), (int32_t)m0);
        for (uint32_t i = pre; i < nkb; i++) {
            const uint32_t s = i % STAGES, round = i / STAGES;
            if (!mbar_wait(&empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY)) break;
            uint8_t *st = smem + s * S::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
            tma_load_2d(st + S::A_BYTES, &p.map_w, &full[s], (int32_t)((kb0 + i) * GEMM_BK),
                        (int32_t)n0);
            tma_load_2d(st, &p.map_a, &full[s], (int32_t)((kb0 + i) * GEMM_BK), (int32_t)m0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: 4 x (128 x BN x 16) per 64-deep K block.
        constexpr uint32_t idesc = umma_idesc_f16(GEMM_BM, BN);
        for (uint32_t i = 0; i < nkb; i++) {
            const uint32_t s = i % STAGES, round = i / STAGES;
            if (!mbar_wait(&full[s], round & 1, JC_DEV_TIMEOUT_FULL)) break;
            tc_fence_after();
            uint8_t *st = smem + s * S::STAGE_BYTES;
            const uint64_t ad = umma_desc_sw128(smem_u32(st));
            const uint64_t bd = umma_desc_sw128(smem_u32(st + S::A_BYTES));
#pragma unroll
            for (uint32_t kk = 0; kk < GEMM_BK / 16; kk++)
                // +32 bytes (2 in descriptor units) per 16-element K step inside the 128B row.
                tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0);
            tc_commit(&empty[s]);
        }
        tc_commit(done);
    }
    __syncwarp();

    // ---- epilogue: warp w owns rows 32(w%4)..+31 and column half w/4 of each chunk ----
    const uint32_t quarter = warp & 3, half = warp >> 2;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t r = m0 + row;
    const bool valid = r < p.m;
    pdl_launch_dependents();
    pdl_wait();

    // Everything the epilogue reads from the previous kernel, fetched while the MMAs run.
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

    // Clear the statistics buffer a later GEMM accumulates into (grid-stride).
    if (p.zero_len) {
        const uint32_t nblk = gridDim.x * gridDim.y * gridDim.z;
        const uint32_t blk = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        for (uint32_t i = blk * GEMM_THREADS + threadIdx.x; i < p.zero_len; i += nblk * GEMM_THREADS)
            p.zero[i] = 0.0f;
    }

    const bool mma_ok = __syncthreads_and(mbar_wait_sleep(done, 0, JC_DEV_TIMEOUT_MMA)) != 0;
    tc_fence_after();
    const uint32_t lane_base = tmem + ((quarter * 32) << 16);
    bool run_epilogue = mma_ok;

    if (splits > 1 && mma_ok) {
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
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
            *last_flag = last ? 1u : 0u;
        }
        __syncthreads();
        run_epilogue = *last_flag != 0;
        __threadfence();
    }

    if (run_epilogue) {
        float s = 0.f, q = 0.f;
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
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
            gemm_epilogue_part<CH, EPI>(p, v, r, valid, n0, la, half, mean, rstd, cs_s, bs_s,
                                        resv + ((EPI & JC_EPI_RES) ? ci * 2 * G / 8 : 0),
                                        ropev + ((EPI & JC_EPI_ROPE) ? ci * 8 : 0), s, q);
        }
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            // The two halves of a row meet in shared memory; one atomic pair per row per tile.
            if (half) row_part[row] = make_float2(s, q);
            __syncthreads();
            if (!half && valid) {
                const float2 o = row_part[row];
                atomicAdd(p.stats_out + 2 * (size_t)r, s + o.x);
                atomicAdd(p.stats_out + 2 * (size_t)r + 1, q + o.y);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

}  // namespace jc
