// The fused-epilogue GEMM for launches of more tiles than SMs (large packs of requests): one CTA
// per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... with its pipeline kept warm across
// them, and the epilogue of one tile overlaps the main loop of the next.
//
//   - warp 0 lane 0 streams every tile's A and W k-blocks through one STAGES-deep TMA ring (no
//     multicast), without waiting for epilogues;
//   - lane 0 of warps 1..NI issue tcgen05.mma (M 128, N BN, K 16) into one of two TMEM
//     accumulator buffers (NI accumulators each, taking the MMAs of a stage round-robin and
//     summed in issuer order, as in gemm_tile.cuh), a buffer reused once the epilogue has read it;
//   - warps 4 and up run the epilogue (persist_tile_epilogue, below): a tile row and a column
//     group of every 64-column chunk a thread, residuals and outputs through a buffer a quarter of
//     the rows;
//   - warp 3 clears the statistics buffer a later GEMM adds into.
// 128-column tiles use two issuers (two 128-wide accumulators a buffer), 256-column tiles one
// (a single N = 256 chain already runs at the tensor pipe's rate): 512 TMEM columns either way.
// Same epilogue arithmetic as gemm.cuh (the reference's, kernels/src/main.rs:931-1037); waits
// bounded as everywhere in this library.
#pragma once
#include "gemm.cuh"

namespace jc {

// ---- the persistent epilogues ----
//
// PERSIST_EPI_CG x 4 epilogue warps (from warp 4): warp w reads TMEM lanes 32 (w % 4) .. + 31
// (its quarter's 32 tile rows, one a thread, as TMEM hands them out) and column group
// g = (w - 4) / 4 of every 64-column chunk: columns [GW g, GW g + GW) and [32 + GW g, 32 + GW g +
// GW) with GW = 32 / PERSIST_EPI_CG, so a thread holds both members of its RoPE pairs (i, i + 32)
// and both the GELU inputs and the gates of its GeGLU outputs. The warps of a quarter share a
// 4 KB buffer of 32 rows x 128 bytes, XOR-swizzled in 16-byte chunks (chunk c of row r at
// c ^ (r & 7): row-per-lane writes and line-per-8-lanes reads are both free of bank conflicts),
// through which residuals come in and outputs go out with 16-byte accesses whose 8 consecutive
// lanes cover one 128-byte row segment. (One row a lane, as TMEM hands them out, touches 32 cache
// lines an instruction: those stores alone cost the 6144-row qkv GEMM a third of its time.) The
// quarter's warps meet at named barrier 1 + quarter. Eight epilogue warps (two to a quarter):
// sixteen (16 columns of a chunk a thread) measured no faster (qkv at 12288 rows 45.1 against
// 45.4 us, wi 47.6 against 46.7, config 3 8093-8191 against 8258-8320 requests/s).
constexpr int PERSIST_EPI_CG = 2;                       // column groups (warps) a quarter
constexpr int PERSIST_EPI_GW = 32 / PERSIST_EPI_CG;     // columns of a half-chunk a thread
constexpr int PERSIST_GEMM_THREADS = 32 * (4 + 4 * PERSIST_EPI_CG);
constexpr int PERSIST_EPI_QUARTER_BYTES = 32 * 128 + PERSIST_EPI_CG * 32 * 8;  // rows, statistics
constexpr int PERSIST_EPI_BYTES = 4 * PERSIST_EPI_QUARTER_BYTES;
static_assert(PERSIST_EPI_GW % 8 == 0, "a thread's columns are whole 16-byte chunks");

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

__device__ __forceinline__ uint4 *quarter_chunk(uint8_t *buf, uint32_t row, uint32_t c) {
    return reinterpret_cast<uint4 *>(buf + row * 128 + ((c ^ (row & 7)) << 4));
}

__device__ __forceinline__ void quarter_sync(uint32_t quarter) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "n"(32 * PERSIST_EPI_CG) : "memory");
}

// quarter_sync that also ANDs a condition over the quarter's warps (so all take the same branch
// after it, and none is left waiting at a later barrier for another).
__device__ __forceinline__ bool quarter_and(uint32_t quarter, bool c) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pc, pr;\n\t"
        "setp.ne.u32 pc, %1, 0;\n\t"
        "bar.red.and.pred pr, %2, %3, pc;\n\t"
        "selp.u32 %0, 1, 0, pr;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)c), "r"(1 + quarter), "n"(32 * PERSIST_EPI_CG)
        : "memory");
    return r != 0;
}

// Rows a warp of a quarter moves in the coalesced loads and stores.
constexpr int PERSIST_EPI_ROWS = 32 / PERSIST_EPI_CG;

// This warp's rows of [row0, row0 + 32) (rows row0 + ROWS g ..) x columns [col, col + 64) of a
// row-major f16 matrix (ld columns a row) into registers, 16 bytes at a time, coalesced (rows from
// `m` on read as zero).
__device__ __forceinline__ void group_load_rows64(const __half *src, uint32_t ld, uint32_t row0,
                                                  uint32_t m, uint32_t col, uint32_t g, uint32_t lane,
                                                  uint4 (&regs)[PERSIST_EPI_ROWS / 4]) {
#pragma unroll
    for (int k = 0; k < PERSIST_EPI_ROWS / 4; k++) {
        const uint32_t r = row0 + PERSIST_EPI_ROWS * g + k * 4 + (lane >> 3);
        regs[k] = r < m ? *reinterpret_cast<const uint4 *>(src + (size_t)r * ld + col + (lane & 7) * 8)
                        : make_uint4(0, 0, 0, 0);
    }
}

// The 16-byte chunks of a 128-byte buffer row a thread of column group g holds: its columns
// [GW g, GW g + GW) and [32 + GW g, 32 + GW g + GW).
__device__ __forceinline__ uint32_t group_chunk(uint32_t g, int j) {
    constexpr int CPS = PERSIST_EPI_GW / 8;  // chunks a segment
    return (uint32_t)((j / CPS) * 4 + CPS * g + (j % CPS));
}

// The residual of a chunk: the quarter's warps put their group_load_rows64 registers in the
// buffer, then every thread takes its columns of its row (GW + GW columns as GW packed words).
__device__ __forceinline__ void quarter_residual(uint8_t *buf, const uint4 (&regs)[PERSIST_EPI_ROWS / 4],
                                                 uint32_t quarter, uint32_t g, uint32_t lane,
                                                 uint32_t *w) {
#pragma unroll
    for (int k = 0; k < PERSIST_EPI_ROWS / 4; k++)
        *quarter_chunk(buf, PERSIST_EPI_ROWS * g + k * 4 + (lane >> 3), lane & 7) = regs[k];
    quarter_sync(quarter);
#pragma unroll
    for (int j = 0; j < PERSIST_EPI_GW / 4; j++) {
        const uint4 t = *quarter_chunk(buf, lane, group_chunk(g, j));
        w[4 * j] = t.x; w[4 * j + 1] = t.y; w[4 * j + 2] = t.z; w[4 * j + 3] = t.w;
    }
}

// A chunk's outputs: every thread puts its words in its row of the buffer (W = 64 output columns a
// row: out[0, GW/2) columns GW g.., out[GW/2, GW) columns 32 + GW g..; W = 32 (GeGLU): out[0,
// GW/2) output columns GW g..), then each warp stores its rows to rows [row0, row0 + 32) x columns
// [col, col + W) of a row-major f16 matrix (ld columns a row; rows from `m` on not written), whole
// row segments at a time. The buffer is free again when this returns.
template <int W>
__device__ __forceinline__ void quarter_store(uint8_t *buf, const uint32_t *out, uint32_t quarter,
                                              uint32_t g, uint32_t lane, __half *dst, uint32_t ld,
                                              uint32_t row0, uint32_t m, uint32_t col) {
    static_assert(W == 64 || W == 32, "64 or 32 output columns a chunk");
    constexpr int NW = (W == 64 ? 2 : 1) * PERSIST_EPI_GW / 8;  // 16-byte pieces a thread
#pragma unroll
    for (int j = 0; j < NW; j++)
        *quarter_chunk(buf, lane, group_chunk(g, j)) =
            make_uint4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
    quarter_sync(quarter);
    constexpr int CH = W / 8;     // 16-byte chunks a row
    constexpr int RPI = 32 / CH;  // rows one instruction covers
#pragma unroll
    for (int k = 0; k < PERSIST_EPI_ROWS / RPI; k++) {
        const uint32_t rr = PERSIST_EPI_ROWS * g + k * RPI + lane / CH, c = lane % CH, r = row0 + rr;
        if (r < m) *reinterpret_cast<uint4 *>(dst + (size_t)r * ld + col + c * 8) = *quarter_chunk(buf, rr, c);
    }
    quarter_sync(quarter);
}

// The epilogue arithmetic of one thread's 2 GW columns of a 64-column chunk starting at
// tile-local column c0 (v[0, GW): columns c0 + GW g + j, v[GW, 2 GW): columns c0 + 32 + GW g + j);
// ropev: (cos, sin) of pairs GW g .. GW g + GW - 1 of the row, two per float4; resw: the residual
// of those columns (GW packed words, RES). Writes GW output words (GW / 2 for GeGLU's GW outputs)
// to out and adds the statistics of the stored values to s / q (STATS).
template <uint32_t EPI>
__device__ __forceinline__ void group_chunk_values(const GemmParams &p, float *v, uint32_t n0,
                                                   uint32_t c0, uint32_t g, float mean, float rstd,
                                                   const float4 *ropev, const uint32_t *resw,
                                                   uint32_t *out, float &s, float &q) {
    constexpr int GW = PERSIST_EPI_GW;
    const uint32_t ga = n0 + c0 + GW * g, gb = ga + 32;
    // Column sums and biases four at a time (ga, gb multiples of 8 columns: 32-byte aligned).
    if constexpr ((EPI & JC_EPI_LN) != 0) {
        const float4 *ca = reinterpret_cast<const float4 *>(p.colsum + ga);
        const float4 *cb = reinterpret_cast<const float4 *>(p.colsum + gb);
#pragma unroll
        for (int j = 0; j < GW / 4; j++) {
            const float4 x = __ldg(ca + j), y = __ldg(cb + j);
            v[4 * j] = rstd * (v[4 * j] - mean * x.x);
            v[4 * j + 1] = rstd * (v[4 * j + 1] - mean * x.y);
            v[4 * j + 2] = rstd * (v[4 * j + 2] - mean * x.z);
            v[4 * j + 3] = rstd * (v[4 * j + 3] - mean * x.w);
            v[GW + 4 * j] = rstd * (v[GW + 4 * j] - mean * y.x);
            v[GW + 4 * j + 1] = rstd * (v[GW + 4 * j + 1] - mean * y.y);
            v[GW + 4 * j + 2] = rstd * (v[GW + 4 * j + 2] - mean * y.z);
            v[GW + 4 * j + 3] = rstd * (v[GW + 4 * j + 3] - mean * y.w);
        }
    }
    if constexpr ((EPI & JC_EPI_BIAS) != 0) {
        const float4 *ba = reinterpret_cast<const float4 *>(p.bias + ga);
        const float4 *bb = reinterpret_cast<const float4 *>(p.bias + gb);
#pragma unroll
        for (int j = 0; j < GW / 4; j++) {
            const float4 x = __ldg(ba + j), y = __ldg(bb + j);
            v[4 * j] += x.x; v[4 * j + 1] += x.y; v[4 * j + 2] += x.z; v[4 * j + 3] += x.w;
            v[GW + 4 * j] += y.x; v[GW + 4 * j + 1] += y.y; v[GW + 4 * j + 2] += y.z; v[GW + 4 * j + 3] += y.w;
        }
    }
    if constexpr ((EPI & JC_EPI_RELU) != 0) {
#pragma unroll
        for (int j = 0; j < 2 * GW; j++) v[j] = fmaxf(v[j], 0.0f);
    }
    if constexpr ((EPI & JC_EPI_GELU) != 0) {
#pragma unroll
        for (int j = 0; j < 2 * GW; j++) v[j] = gelu_as(v[j]);
    }
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        // q and k are the first two thirds of a qkv row; the chunk is one head.
        if (n0 + c0 < 2 * (p.n / 3)) {
#pragma unroll
            for (int j = 0; j < GW; j++) {
                const float4 t = ropev[j / 2];
                const float c = (j & 1) ? t.z : t.x, sn = (j & 1) ? t.w : t.y;
                const float x1 = v[j], x2 = v[GW + j];
                v[j] = x1 * c - x2 * sn;
                v[GW + j] = x2 * c + x1 * sn;
            }
        }
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
        // Columns c0 .. c0 + 31 of the chunk are GELU inputs of outputs (c0 / 2) .. + 31, the next
        // 32 their gates: this thread's GW inputs and GW gates give outputs GW g ...
#pragma unroll
        for (int j = 0; j < GW / 2; j++)
            out[j] = pack_half2(gelu_as(v[2 * j]) * v[GW + 2 * j], gelu_as(v[2 * j + 1]) * v[GW + 2 * j + 1]);
    } else {
        pack_group<GW, EPI>(v, resw, out, s, q);
        pack_group<GW, EPI>(v + GW, resw + GW / 2, out + GW / 2, s, q);
    }
}

// One tile's epilogue by one thread of the epilogue warps (quarter, column group g, lane): its row
// m0 + 32 quarter + lane of the tile, columns n0 .. n0 + BN, the accumulator at TMEM address acc
// (this warp's lanes; NI accumulators BN columns apart, summed in issuer order) once `acc_full`
// completes its phase of this parity. `release` runs on lane 0 of each warp after the warp's last
// TMEM read of the tile. qbuf: the quarter's buffer, its statistics slots after the 32 rows.
// false if the accumulator wait gave up.
template <int BN, int NI, uint32_t EPI, class Release>
__device__ __forceinline__ bool persist_tile_epilogue(const GemmParams &p, uint32_t acc, uint64_t *acc_full,
                                                      uint32_t parity, uint8_t *qbuf, uint32_t quarter,
                                                      uint32_t g, uint32_t lane, uint32_t m0,
                                                      uint32_t n0, Release release) {
    constexpr int GW = PERSIST_EPI_GW;
    const uint32_t row0 = m0 + quarter * 32, r = row0 + lane;
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
    constexpr int ROPE_V = (EPI & JC_EPI_ROPE) ? GW / 2 : 1;
    float4 ropev[ROPE_V];
#pragma unroll
    for (int i = 0; i < ROPE_V; i++) ropev[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr ((EPI & JC_EPI_ROPE) != 0) {
        if (valid) {
            // Pair-group-major table: float4 k holds pairs 2k, 2k + 1 of every row.
            const uint32_t pos = p.seg ? r - p.seg[r].x : r;
            const float4 *t4 = reinterpret_cast<const float4 *>(p.rope) + (size_t)(GW / 2 * g) * p.rope_stride + pos;
#pragma unroll
            for (int i = 0; i < GW / 2; i++) ropev[i] = __ldg(t4 + (size_t)i * p.rope_stride);
        }
    }
    uint4 res[PERSIST_EPI_ROWS / 4];
    if constexpr ((EPI & JC_EPI_RES) != 0) group_load_rows64(p.res, p.n, row0, p.m, n0, g, lane, res);
    if (!quarter_and(quarter, mbar_wait_sleep(acc_full, parity, JC_DEV_TIMEOUT_MMA))) return false;
    tc_fence_after();
    float s = 0.f, q = 0.f;
    // A chunk's accumulator columns are requested while the chunk before it is processed: two
    // register sets, alternating (the loop is unrolled, so both stay in registers).
    constexpr int CHUNKS = BN / 64;
    float vv[2][2 * GW];
    float tt[2][NI > 1 ? 2 * GW : 1];
    auto request = [&](uint32_t ci, int b) {
        const uint32_t col = acc + ci * 64 + GW * g;
        tmem_ld<GW>(col, vv[b]);
        tmem_ld<GW>(col + 32, vv[b] + GW);
        if constexpr (NI > 1) {
            tmem_ld<GW>(col + BN, tt[b]);
            tmem_ld<GW>(col + BN + 32, tt[b] + GW);
        }
    };
    request(0, 0);
#pragma unroll
    for (uint32_t ci = 0; ci < (uint32_t)CHUNKS; ci++) {
        const int b = ci & 1;
        tc_wait_ld();
        if (ci + 1 < (uint32_t)CHUNKS) {
            request(ci + 1, b ^ 1);
        } else {
            // This warp has read every column of the buffer it reads.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release();
        }
        float *v = vv[b];
        if constexpr (NI > 1) {
#pragma unroll
            for (int e = 0; e < 2 * GW; e++) v[e] += tt[b][e];
        }
        uint32_t resw[GW];
        if constexpr ((EPI & JC_EPI_RES) != 0) {
            quarter_residual(qbuf, res, quarter, g, lane, resw);
            if (ci + 1 < (uint32_t)BN / 64) group_load_rows64(p.res, p.n, row0, p.m, n0 + (ci + 1) * 64, g, lane, res);
        }
        uint32_t out[GW];
        float s1 = 0.f, q1 = 0.f;
        group_chunk_values<EPI>(p, v, n0, ci * 64, g, mean, rstd, ropev, resw, out, s1, q1);
        s += s1;
        q += q1;
        if constexpr ((EPI & JC_EPI_GEGLU) != 0)
            quarter_store<32>(qbuf, out, quarter, g, lane, p.c, p.n / 2, row0, p.m, (n0 + ci * 64) / 2);
        else
            quarter_store<64>(qbuf, out, quarter, g, lane, p.c, p.n, row0, p.m, n0 + ci * 64);
    }
    if constexpr ((EPI & JC_EPI_STATS) != 0) {
        // The row's column groups meet in the quarter's statistics slots: one atomic pair a row.
        float2 *st = reinterpret_cast<float2 *>(qbuf + 32 * 128);
        if (g) st[(g - 1) * 32 + lane] = make_float2(s, q);
        quarter_sync(quarter);
        if (!g && valid) {
#pragma unroll
            for (int k = 0; k < PERSIST_EPI_CG - 1; k++) {
                const float2 o = st[k * 32 + lane];
                s += o.x;
                q += o.y;
            }
            red_add_f32x2(p.stats_out + 2 * (size_t)r, s, q);
        }
    }
    return true;
}

template <int BN, int STAGES, uint32_t EPI>
__global__ void __launch_bounds__(PERSIST_GEMM_THREADS, 1)
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
            mbar_init(&acc_empty[b], 4 * PERSIST_EPI_CG);  // lane 0 of each epilogue warp
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
        // Epilogue (4 PERSIST_EPI_CG warps; with one issuer, warp 2 has no role and idles).
        pdl_wait();
        pdl_launch_dependents();
        const uint32_t quarter = warp & 3, grp = (warp - 4) >> 2;
        const uint32_t lane_base = tmem + ((quarter * 32) << 16);
        uint8_t *qbuf = base + S::EPI_OFF + quarter * PERSIST_EPI_QUARTER_BYTES;
        for (uint32_t t = blockIdx.x, i = 0; t < total; t += gridDim.x, i++) {
            const uint32_t buf = i & 1;
            const uint32_t m0 = (t / tiles_n) * GEMM_BM, n0 = (t % tiles_n) * BN;
            // The MMAs of the tile after next may overwrite this buffer once every epilogue warp has
            // read its part.
            if (!persist_tile_epilogue<BN, NI, EPI>(p, lane_base + buf * S::ACC, &acc_full[buf], (i >> 1) & 1,
                                                    qbuf, quarter, grp, lane, m0, n0,
                                                    [&] { mbar_arrive(&acc_empty[buf]); }))
                break;
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
