// The fused-epilogue GEMM for launches of more tiles than SMs (large packs of requests): one CTA
// per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... with its pipeline kept warm across
// them, and the epilogue of one tile overlaps the main loop of the next.
//
//   - warp 0 lane 0 streams every tile's A and W k-blocks through one STAGES-deep TMA ring (no
//     multicast), without waiting for epilogues;
//   - lane 0 of warps 1..NI issue tcgen05.mma (M 128, N BN, K 16) into one of two TMEM
//     accumulator buffers (NI accumulators each, taking the MMAs of a stage round-robin and
//     summed in issuer order, as in gemm_tile.cuh), a buffer reused once the epilogue has read it;
//   - warps 4-7 run the epilogue, one tile row per thread, 64 columns at a time (RoPE pairs
//     (i, i + 32) and GeGLU input / gate pairs stay inside a thread); residuals come in and
//     outputs go out through a 4 KB buffer a warp, so 8 lanes move one 128-byte row segment (one
//     row a lane, as TMEM hands them out, touched 32 cache lines an instruction: the stores alone
//     cost the 6144-row qkv GEMM a third of its time);
//   - warp 3 clears the statistics buffer a later GEMM adds into.
// 128-column tiles use two issuers (two 128-wide accumulators a buffer), 256-column tiles one
// (a single N = 256 chain already runs at the tensor pipe's rate): 512 TMEM columns either way.
// Same epilogue arithmetic as gemm.cuh (the reference's, kernels/src/main.rs:931-1037); waits
// bounded as everywhere in this library.
#pragma once
#include "gemm.cuh"

namespace jc {

// ---- the persistent epilogues' output path ----
//
// Each epilogue warp owns 32 tile rows (one a thread, as TMEM hands them out) and a 4 KB
// shared-memory buffer of 32 rows x 128 bytes, XOR-swizzled in 16-byte chunks (chunk c of row r at
// c ^ (r & 7): a warp's row-per-lane writes and its line-per-8-lanes reads are both free of bank
// conflicts). Residuals come in and outputs go out through it with 16-byte accesses whose 8
// consecutive lanes cover one 128-byte row segment, instead of one row (one cache line) a lane.
constexpr int PERSIST_EPI_WARP_BYTES = 32 * 128;
constexpr int PERSIST_EPI_BYTES = 4 * PERSIST_EPI_WARP_BYTES;

template <int BN, int STAGES_>
struct GemmPersistShape {
    static constexpr int STAGES = STAGES_;
    static constexpr int NI = BN >= 256 ? 1 : 2;
    static constexpr int ACC = NI * BN;  // columns of one accumulator buffer
    static constexpr int A_KB = GEMM_BM * GEMM_BK * 2;
    static constexpr int W_KB = BN * GEMM_BK * 2;
    static constexpr int A_BYTES = GEMM_KPS * A_KB;
    static constexpr int STAGE_BYTES = A_BYTES + GEMM_KPS * W_KB;
    // stages | barriers (1 KB) | the epilogue warps' buffers
    static constexpr int EPI_OFF = STAGES * STAGE_BYTES + 1024;
    static constexpr int SMEM_BYTES = EPI_OFF + PERSIST_EPI_BYTES;
    static_assert(2 * ACC <= 512, "two accumulator buffers in TMEM");
    static_assert(STAGE_BYTES % 1024 == 0, "stages keep 1024-byte alignment");
};

__device__ __forceinline__ uint4 *warp_buf_chunk(uint8_t *buf, uint32_t row, uint32_t c) {
    return reinterpret_cast<uint4 *>(buf + row * 128 + ((c ^ (row & 7)) << 4));
}

// Rows [row0, row0 + 32) x columns [col, col + 64) of a row-major f16 matrix (ld columns a row)
// into registers, 8 x 16 bytes a lane (rows from `m` on read as zero).
__device__ __forceinline__ void warp_load_rows64(const __half *src, uint32_t ld, uint32_t row0,
                                                 uint32_t m, uint32_t col, uint32_t lane,
                                                 uint4 (&regs)[8]) {
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t r = row0 + k * 4 + (lane >> 3);
        regs[k] = r < m ? *reinterpret_cast<const uint4 *>(src + (size_t)r * ld + col + (lane & 7) * 8)
                        : make_uint4(0, 0, 0, 0);
    }
}

// warp_load_rows64's registers into the buffer, then this lane's own row (lane) out of it as 32
// packed half2 words.
__device__ __forceinline__ void warp_rows_to_lane(uint8_t *buf, const uint4 (&regs)[8], uint32_t lane,
                                                  uint32_t *row_words) {
#pragma unroll
    for (int k = 0; k < 8; k++) *warp_buf_chunk(buf, k * 4 + (lane >> 3), lane & 7) = regs[k];
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint4 t = *warp_buf_chunk(buf, lane, j);
        row_words[4 * j] = t.x; row_words[4 * j + 1] = t.y; row_words[4 * j + 2] = t.z; row_words[4 * j + 3] = t.w;
    }
    __syncwarp();
}

// This lane's row of W f16 outputs (W / 2 packed words, W = 64 or 32) into the buffer, then the
// warp's 32 rows to rows [row0, row0 + 32) x columns [col, col + W) of a row-major f16 matrix (ld
// columns a row; rows from `m` on are not written).
template <int W>
__device__ __forceinline__ void warp_store_rows(uint8_t *buf, const uint32_t *row_words, uint32_t lane,
                                                __half *dst, uint32_t ld, uint32_t row0, uint32_t m,
                                                uint32_t col) {
    static_assert(W == 64 || W == 32, "64- or 32-column rows");
    constexpr int CH = W / 8;  // 16-byte chunks a row
#pragma unroll
    for (int j = 0; j < CH; j++)
        *warp_buf_chunk(buf, lane, j) = make_uint4(row_words[4 * j], row_words[4 * j + 1],
                                                   row_words[4 * j + 2], row_words[4 * j + 3]);
    __syncwarp();
    constexpr int RPI = 32 / CH;  // rows one instruction covers
#pragma unroll
    for (int k = 0; k < 32 / RPI; k++) {
        const uint32_t rr = k * RPI + lane / CH, c = lane % CH, r = row0 + rr;
        if (r < m) *reinterpret_cast<uint4 *>(dst + (size_t)r * ld + col + c * 8) = *warp_buf_chunk(buf, rr, c);
    }
    __syncwarp();
}

// The epilogue arithmetic of columns [c0, c0 + 64) (tile-local, c0 a multiple of 64) of one tile
// row, held by one thread: v[64] the accumulator; ropev: (cos, sin) of the row's 32 pairs, two per
// float4; resw: the residual of those columns (32 packed words, RES epilogues). Writes the output
// words to `out` (32, or 16 for GeGLU's 32 output columns) and adds the statistics of the stored
// values to s / q (STATS epilogues).
template <uint32_t EPI>
__device__ __forceinline__ void row_chunk_values(const GemmParams &p, float *v, uint32_t n0,
                                                 uint32_t c0, float mean, float rstd,
                                                 const float4 *ropev, const uint32_t *resw,
                                                 uint32_t *out, float &s, float &q) {
    const uint32_t gc = n0 + c0;
    if constexpr ((EPI & JC_EPI_LN) != 0) {
#pragma unroll
        for (int j = 0; j < 64; j++) v[j] = rstd * (v[j] - mean * __ldg(p.colsum + gc + j));
    }
    if constexpr ((EPI & JC_EPI_BIAS) != 0) {
#pragma unroll
        for (int j = 0; j < 64; j++) v[j] += __ldg(p.bias + gc + j);
    }
    if constexpr ((EPI & JC_EPI_RELU) != 0) {
#pragma unroll
        for (int j = 0; j < 64; j++) v[j] = fmaxf(v[j], 0.0f);
    }
    if constexpr ((EPI & JC_EPI_GELU) != 0) {
#pragma unroll
        for (int j = 0; j < 64; j++) v[j] = gelu_as(v[j]);
    }
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        // q and k are the first two thirds of a qkv row; the chunk is one head.
        if (gc < 2 * (p.n / 3)) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float4 t = ropev[i / 2];
                const float c = (i & 1) ? t.z : t.x, sn = (i & 1) ? t.w : t.y;
                const float x1 = v[i], x2 = v[i + 32];
                v[i] = x1 * c - x2 * sn;
                v[i + 32] = x2 * c + x1 * sn;
            }
        }
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
        // Packed columns [gc, gc + 32) are GELU inputs of output columns [gc/2, gc/2 + 32), the
        // next 32 their gates.
#pragma unroll
        for (int j = 0; j < 16; j++)
            out[j] = pack_half2(gelu_as(v[2 * j]) * v[32 + 2 * j], gelu_as(v[2 * j + 1]) * v[32 + 2 * j + 1]);
    } else {
        pack_group<64, EPI>(v, resw, out, s, q);
    }
}

// The epilogue of one 64-column accumulator chunk of a persistent kernel's tile, by one warp (its
// 32 rows from row0, this lane's row r valid or not): the residual (RES: staged in `res` by the
// caller, the warp's registers from warp_load_rows64) through the buffer, the arithmetic, and the
// outputs through the buffer to c.
template <uint32_t EPI>
__device__ __forceinline__ void persist_chunk_epilogue(const GemmParams &p, float *v, uint8_t *buf,
                                                       const uint4 (&res)[8], uint32_t lane,
                                                       uint32_t row0, bool valid, uint32_t n0,
                                                       uint32_t c0, float mean, float rstd,
                                                       const float4 *ropev, float &s, float &q) {
    uint32_t resw[32];
    if constexpr ((EPI & JC_EPI_RES) != 0) warp_rows_to_lane(buf, res, lane, resw);
    uint32_t out[32];
    float s1 = 0.f, q1 = 0.f;
    row_chunk_values<EPI>(p, v, n0, c0, mean, rstd, ropev, resw, out, s1, q1);
    if (valid) {
        s += s1;
        q += q1;
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0)
        warp_store_rows<32>(buf, out, lane, p.c, p.n / 2, row0, p.m, (n0 + c0) / 2);
    else
        warp_store_rows<64>(buf, out, lane, p.c, p.n, row0, p.m, n0 + c0);
}

template <int BN, int STAGES, uint32_t EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_persistent_kernel(const __grid_constant__ GemmKernelParams kp) {
    dev_err_bind(kp.p.err);
    using S = GemmPersistShape<BN, STAGES>;
    constexpr int NI = S::NI;
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

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NI);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], NI);
            mbar_init(&acc_empty[b], 4);  // lane 0 of each epilogue warp
        }
        fence_barrier_init();
    }
    if (threadIdx.x == 32) {
        tma_prefetch_desc(p.map_a);
        tma_prefetch_desc(p.map_w);
    }
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const uint32_t tiles_n = p.n / BN, tiles_m = (p.m + GEMM_BM - 1) / GEMM_BM;
    const uint32_t total = tiles_m * tiles_n, nst = gemm_stages(p.k / GEMM_BK);

    if (warp == 0) {
        if (lane == 0) {
            // The first stage's weights are requested before the previous kernel has finished.
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x, i = 0; ok && t < total; t += gridDim.x, i++) {
                const uint32_t m0 = (t / tiles_n) * GEMM_BM, n0 = (t % tiles_n) * BN;
                for (uint32_t st = 0; st < nst; st++, g++) {
                    const uint32_t s = g % STAGES, round = g / STAGES;
                    if (round > 0 && !mbar_wait(&empty[s], (round & 1) ^ 1, JC_DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *stage = base + s * S::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
                    tma_load_3d(stage + S::A_BYTES, p.map_w, &full[s], 0, (int32_t)n0, (int32_t)(st * GEMM_KPS));
                    if (g == 0) {
                        pdl_wait();
                        pdl_launch_dependents();
                    }
                    tma_load_3d(stage, p.map_a, &full[s], 0, (int32_t)m0, (int32_t)(st * GEMM_KPS));
                }
            }
        }
    } else if (warp >= 1 && warp <= (uint32_t)NI) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(GEMM_BM, BN);
            const uint32_t j = warp - 1;
            const uint32_t kbs_total = p.k / GEMM_BK;
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x, i = 0; ok && t < total; t += gridDim.x, i++) {
                const uint32_t buf = i & 1, acc = tmem + buf * S::ACC + j * BN;
                // The epilogue has read this buffer's previous tile (two tiles ago).
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
                    for (uint32_t qq = j; qq < 4 * GEMM_KPS; qq += NI) {
                        const uint32_t kb = qq / 4, kk = qq % 4;
                        if (kb < kbs) {
                            const uint64_t ad = umma_desc_sw128(smem_u32(stage + kb * S::A_KB));
                            const uint64_t bd = umma_desc_sw128(smem_u32(stage + S::A_BYTES + kb * S::W_KB));
                            tc_mma_f16(acc, ad + 2 * kk, bd + 2 * kk, idesc, started);
                            started = true;
                        }
                    }
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&acc_full[buf]);
            }
        }
    } else if (warp == 3) {
        pdl_wait();
        pdl_launch_dependents();
        // This warp alone clears the buffer, striding over every CTA's warp 3.
        for (uint32_t i = blockIdx.x * 32 + lane; i < p.zero_len; i += gridDim.x * 32) p.zero[i] = 0.0f;
    } else if (warp >= 4) {
        // Epilogue: warp w reads TMEM lanes 32 (w - 4) .. + 31, one tile row per thread. (With
        // one issuer, warp 2 has no role and idles.)
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t quarter = warp - 4, row = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((quarter * 32) << 16);
        uint8_t *wbuf = base + S::EPI_OFF + quarter * PERSIST_EPI_WARP_BYTES;
        for (uint32_t t = blockIdx.x, i = 0; t < total; t += gridDim.x, i++) {
            const uint32_t buf = i & 1;
            const uint32_t m0 = (t / tiles_n) * GEMM_BM, n0 = (t % tiles_n) * BN;
            const uint32_t r = m0 + row;
            const bool valid = r < p.m;
            // What the epilogue reads besides the accumulator, requested before waiting for it.
            float mean = 0.f, rstd = 0.f;
            if constexpr ((EPI & JC_EPI_LN) != 0) {
                if (valid) {
                    const float2 st = *reinterpret_cast<const float2 *>(p.stats_in + 2 * (size_t)r);
                    mean = st.x / (float)p.k;
                    rstd = rsqrtf(fmaxf(st.y / (float)p.k - mean * mean, 0.0f) + p.eps);
                }
            }
            constexpr int ROPE_V = (EPI & JC_EPI_ROPE) ? 16 : 1;
            float4 ropev[ROPE_V];
#pragma unroll
            for (int g4 = 0; g4 < ROPE_V; g4++) ropev[g4] = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr ((EPI & JC_EPI_ROPE) != 0) {
                if (valid) {
                    const uint32_t pos = p.seg ? r - p.seg[r].x : r;
                    const float4 *t4 = reinterpret_cast<const float4 *>(p.rope) + pos;
#pragma unroll
                    for (int g4 = 0; g4 < 16; g4++) ropev[g4] = __ldg(t4 + (size_t)g4 * p.rope_stride);
                }
            }
            // The first chunk's residual rows (coalesced, through this warp's buffer later).
            const uint32_t row0 = m0 + quarter * 32;
            uint4 res[8];
            if constexpr ((EPI & JC_EPI_RES) != 0) warp_load_rows64(p.res, p.n, row0, p.m, n0, lane, res);
            if (!mbar_wait_sleep(&acc_full[buf], (i >> 1) & 1, JC_DEV_TIMEOUT_MMA)) break;
            tc_fence_after();
            float s = 0.f, q = 0.f;
#pragma unroll 1
            for (uint32_t ci = 0; ci < (uint32_t)BN / 64; ci++) {
                float v[64];
                const uint32_t col = lane_base + buf * S::ACC + ci * 64;
#pragma unroll
                for (int c = 0; c < 4; c++) tmem_ld<16>(col + 16 * c, v + 16 * c);
                if constexpr (NI > 1) {
                    float t2[64];
#pragma unroll
                    for (int c = 0; c < 4; c++) tmem_ld<16>(col + BN + 16 * c, t2 + 16 * c);
                    tc_wait_ld();
#pragma unroll
                    for (int e = 0; e < 64; e++) v[e] += t2[e];
                } else {
                    tc_wait_ld();
                }
                if (ci == (uint32_t)BN / 64 - 1) {
                    // Every column of this buffer is read: the MMAs of the tile after next may
                    // overwrite it.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                }
                persist_chunk_epilogue<EPI>(p, v, wbuf, res, lane, row0, valid, n0, ci * 64, mean, rstd,
                                            ropev, s, q);
                // The next chunk's residual rows.
                if constexpr ((EPI & JC_EPI_RES) != 0)
                    if (ci + 1 < (uint32_t)BN / 64) warp_load_rows64(p.res, p.n, row0, p.m, n0 + (ci + 1) * 64, lane, res);
            }
            if constexpr ((EPI & JC_EPI_STATS) != 0) {
                if (valid) red_add_f32x2(p.stats_out + 2 * (size_t)r, s, q);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace jc
