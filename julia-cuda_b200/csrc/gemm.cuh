// The encoder's fused-epilogue GEMM family on sm_100a tensor cores.
//
// c = epilogue(a . w^T): a [m, k] f16 row-major (activations), w [n, k] f16 row-major (nn.Linear
// weights), f32 accumulation in tensor memory. Replaces the reference's mma.sync family
// (kernels/src/gemm.rs:317-433 mainloop / split_reduce, kernels/src/main.rs:886-1147 gemm_tile
// and its 32 instances) with one tcgen05 design:
//
//   - a CTA computes a 128 x BN tile (BN = 32, 64 or 128) with 128 threads;
//   - warp 0 lane 0 streams 64-deep K blocks of A and W into a STAGES-deep ring of 128B-swizzled
//     shared-memory tiles with TMA (no multicast), each stage completing on an mbarrier;
//   - warp 1 lane 0 issues tcgen05.mma (M=128, N=BN, K=16, kind::f16) into a TMEM accumulator and
//     releases each stage with tcgen05.commit;
//   - all four warps run the epilogue: thread t owns tile row t (TMEM lane t), loads its row with
//     tcgen05.ld and applies the fused epilogue in registers.
//
// Because one thread holds a whole row of the tile, the RoPE pairs (i, i + 32) of a 64-column head
// and the row statistics need no shuffles: q and k stay in natural (checkpoint) order, and GeGLU
// only needs Wi's rows interleaved in blocks of 32 (prep_interleave_geglu), not the reference's
// fragment-level permutations (src/prep.rs:67-101).
//
// Split-K (gridDim.z > 1): every split stores its f32 partial tile to `ws`, the last split of a
// tile to arrive (atomic counter, reset by it) sums all partials in split order, so the result
// does not depend on arrival order (the reference's scheme, src/gemm.rs:364-433), then runs the
// epilogue.
//
// Programmatic dependent launch: the weight tiles of the first stages are requested before
// griddepcontrol.wait, so they stream in while the previous kernel drains; activations, statistics
// and residuals are read only after it.
#pragma once
#include "common.cuh"

namespace jc {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 128;
constexpr int GEMM_STAGES = 4;

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

template <int BN>
struct GemmShape {
    static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
    static constexpr int B_BYTES = BN * GEMM_BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int CH = BN < 64 ? BN : 64;  // epilogue chunk (columns in registers)
    static constexpr int SMEM_BYTES = GEMM_STAGES * STAGE_BYTES + 1024 /* align */ + 256;
    static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
};

// One epilogue chunk of CH columns for row r (valid = r < m), starting at packed column c0.
template <int CH, uint32_t EPI>
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmParams &p, float (&v)[CH],
                                                    uint32_t r, bool valid, uint32_t c0,
                                                    float mean, float rstd, float &s, float &q) {
    if constexpr ((EPI & JC_EPI_LN) != 0) {
        const float4 *cs = reinterpret_cast<const float4 *>(p.colsum + c0);
#pragma unroll
        for (int j = 0; j < CH / 4; j++) {
            float4 c4 = __ldg(cs + j);
            v[4 * j + 0] = rstd * (v[4 * j + 0] - mean * c4.x);
            v[4 * j + 1] = rstd * (v[4 * j + 1] - mean * c4.y);
            v[4 * j + 2] = rstd * (v[4 * j + 2] - mean * c4.z);
            v[4 * j + 3] = rstd * (v[4 * j + 3] - mean * c4.w);
        }
    }
    if constexpr ((EPI & JC_EPI_BIAS) != 0) {
        const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + c0);
#pragma unroll
        for (int j = 0; j < CH / 4; j++) {
            float4 b = __ldg(b4 + j);
            v[4 * j + 0] += b.x;
            v[4 * j + 1] += b.y;
            v[4 * j + 2] += b.z;
            v[4 * j + 3] += b.w;
        }
    }
    if constexpr ((EPI & JC_EPI_RELU) != 0) {
#pragma unroll
        for (int j = 0; j < CH; j++) v[j] = fmaxf(v[j], 0.0f);
    }
    if constexpr ((EPI & JC_EPI_GELU) != 0) {
#pragma unroll
        for (int j = 0; j < CH; j++) v[j] = gelu_as(v[j]);
    }
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        static_assert(CH == 64, "RoPE needs whole 64-column heads");
        // q and k are the first two thirds of a qkv row; the chunk is exactly one head.
        if (valid && c0 < 2 * (p.n / 3)) {
            const float4 *t4 = reinterpret_cast<const float4 *>(p.rope + (size_t)r * 64);
#pragma unroll
            for (int i = 0; i < 16; i++) {
                float4 t = __ldg(t4 + i);  // (cos, sin) of pairs 2i and 2i + 1
                float x1 = v[2 * i], x2 = v[2 * i + 32];
                v[2 * i] = x1 * t.x - x2 * t.y;
                v[2 * i + 32] = x2 * t.x + x1 * t.y;
                x1 = v[2 * i + 1];
                x2 = v[2 * i + 33];
                v[2 * i + 1] = x1 * t.z - x2 * t.w;
                v[2 * i + 33] = x2 * t.z + x1 * t.w;
            }
        }
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
        static_assert(CH == 64, "GeGLU needs 32 input and 32 gate columns per chunk");
        if (valid) {
            // Packed columns [c0, c0 + 32) are GELU inputs of output columns [c0/2, c0/2 + 32),
            // [c0 + 32, c0 + 64) their gates.
            uint4 *dst = reinterpret_cast<uint4 *>(p.c + (size_t)r * (p.n / 2) + c0 / 2);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint4 o;
                o.x = pack_half2(gelu_as(v[8 * j + 0]) * v[8 * j + 32],
                                 gelu_as(v[8 * j + 1]) * v[8 * j + 33]);
                o.y = pack_half2(gelu_as(v[8 * j + 2]) * v[8 * j + 34],
                                 gelu_as(v[8 * j + 3]) * v[8 * j + 35]);
                o.z = pack_half2(gelu_as(v[8 * j + 4]) * v[8 * j + 36],
                                 gelu_as(v[8 * j + 5]) * v[8 * j + 37]);
                o.w = pack_half2(gelu_as(v[8 * j + 6]) * v[8 * j + 38],
                                 gelu_as(v[8 * j + 7]) * v[8 * j + 39]);
                dst[j] = o;
            }
        }
    } else {
        if (valid) {
            uint4 *dst = reinterpret_cast<uint4 *>(p.c + (size_t)r * p.n + c0);
            const uint4 *src = reinterpret_cast<const uint4 *>(p.res + (size_t)r * p.n + c0);
#pragma unroll
            for (int j = 0; j < CH / 8; j++) {
                float w[8];
#pragma unroll
                for (int e = 0; e < 8; e++) w[e] = v[8 * j + e];
                if constexpr ((EPI & JC_EPI_RES) != 0) {
                    // res may alias c: each thread reads only the values it overwrites next.
                    uint4 rr = src[j];
                    float2 a = unpack_half2(rr.x), b = unpack_half2(rr.y);
                    float2 cc = unpack_half2(rr.z), d = unpack_half2(rr.w);
                    w[0] += a.x; w[1] += a.y; w[2] += b.x; w[3] += b.y;
                    w[4] += cc.x; w[5] += cc.y; w[6] += d.x; w[7] += d.y;
                }
                uint4 o;
                o.x = pack_half2(w[0], w[1]);
                o.y = pack_half2(w[2], w[3]);
                o.z = pack_half2(w[4], w[5]);
                o.w = pack_half2(w[6], w[7]);
                dst[j] = o;
                if constexpr ((EPI & JC_EPI_STATS) != 0) {
                    // Statistics of the values as stored (f16), as the next LayerNorm sees them.
                    const uint32_t pk[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        float2 f = unpack_half2(pk[e]);
                        s += f.x + f.y;
                        q = fmaf(f.x, f.x, q);
                        q = fmaf(f.y, f.y, q);
                    }
                }
            }
        }
    }
}

template <int BN, uint32_t EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    using S = GemmShape<BN>;
    constexpr int CH = S::CH;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + GEMM_STAGES * S::STAGE_BYTES);
    uint64_t *empty = full + GEMM_STAGES;
    uint64_t *done = empty + GEMM_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    uint32_t *last_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * GEMM_BM;
    const uint32_t z = blockIdx.z, splits = gridDim.z;
    const uint32_t kb_total = p.k / GEMM_BK;
    const uint32_t kb0 = z * kb_total / splits, kb1 = (z + 1) * kb_total / splits;
    const uint32_t nkb = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GEMM_STAGES; s++) {
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
    if (warp == 0) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer. The weight tiles of the first stages do not depend on the previous
        // kernel: request them before waiting for it.
        const uint32_t pre = nkb < (uint32_t)GEMM_STAGES ? nkb : (uint32_t)GEMM_STAGES;
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
            const uint32_t s = i % GEMM_STAGES, round = i / GEMM_STAGES;
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
            const uint32_t s = i % GEMM_STAGES, round = i / GEMM_STAGES;
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

    // ---- epilogue: thread t owns row m0 + t (TMEM lane t) ----
    pdl_launch_dependents();
    const bool mma_ok = mbar_wait(done, 0, JC_DEV_TIMEOUT_MMA);
    tc_fence_after();
    pdl_wait();

    // Clear the statistics buffer a later GEMM accumulates into (grid-stride).
    if (p.zero_len) {
        const uint32_t nblk = gridDim.x * gridDim.y * gridDim.z;
        const uint32_t blk = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        for (uint32_t i = blk * GEMM_THREADS + threadIdx.x; i < p.zero_len; i += nblk * GEMM_THREADS)
            p.zero[i] = 0.0f;
    }

    const uint32_t row = warp * 32 + lane;
    const uint32_t r = m0 + row;
    const bool valid = r < p.m;
    const uint32_t lane_base = tmem + ((warp * 32) << 16);
    bool run_epilogue = mma_ok;

    if (splits > 1 && mma_ok) {
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
        float *mine = p.ws + ((size_t)tile * splits + z) * BN * GEMM_BM;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(lane_base + c, v);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j++) mine[(size_t)(c + j) * GEMM_BM + row] = v[j];
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
        float mean = 0.f, rstd = 0.f;
        if constexpr ((EPI & JC_EPI_LN) != 0) {
            if (valid) {
                const float2 st = *reinterpret_cast<const float2 *>(p.stats_in + 2 * (size_t)r);
                mean = st.x / (float)p.k;
                float var = st.y / (float)p.k - mean * mean;
                rstd = rsqrtf(fmaxf(var, 0.0f) + p.eps);
            }
        }
        float s = 0.f, q = 0.f;
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
#pragma unroll 1
        for (int cb = 0; cb < BN; cb += CH) {
            float v[CH];
            if (splits == 1) {
#pragma unroll
                for (int h = 0; h < CH; h += 32) {
                    float t[32];
                    tmem_ld32(lane_base + cb + h, t);
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j++) v[h + j] = t[j];
                }
            } else {
#pragma unroll
                for (int j = 0; j < CH; j++) v[j] = 0.0f;
                for (uint32_t zz = 0; zz < splits; zz++) {
                    if (zz == z) {
#pragma unroll
                        for (int h = 0; h < CH; h += 32) {
                            float t[32];
                            tmem_ld32(lane_base + cb + h, t);
                            tc_wait_ld();
#pragma unroll
                            for (int j = 0; j < 32; j++) v[h + j] += t[j];
                        }
                    } else {
                        const float *part = p.ws + ((size_t)tile * splits + zz) * BN * GEMM_BM;
#pragma unroll
                        for (int j = 0; j < CH; j++)
                            v[j] += __ldcg(part + (size_t)(cb + j) * GEMM_BM + row);
                    }
                }
            }
            gemm_epilogue_chunk<CH, EPI>(p, v, r, valid, n0 + cb, mean, rstd, s, q);
        }
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            if (valid) {
                atomicAdd(p.stats_out + 2 * (size_t)r, s);
                atomicAdd(p.stats_out + 2 * (size_t)r + 1, q);
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
