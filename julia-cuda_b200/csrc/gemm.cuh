// The encoder's fused-epilogue GEMM family on sm_100a tensor cores.
//
// c = epilogue(a . w^T): a [m, k] f16 row-major (activations), w [n, k] f16 row-major (nn.Linear
// weights), f32 accumulation in tensor memory. Replaces the reference's mma.sync family
// (kernels/src/gemm.rs:317-433 mainloop / split_reduce, kernels/src/main.rs:886-1147 gemm_tile
// and its 32 instances) with one tcgen05 design:
//
//   - a CTA computes a BM x BN tile (BM = 128, or 64 for narrow GEMMs at a few hundred rows: half
//     the activation bytes a CTA ingests, which bounds the main loop; BN = 32, 64, 128 or 256)
//     with 256 threads;
//   - warp 0 lane 0 streams 64-deep K blocks of A and W into a ring of STAGES 128B-swizzled
//     shared-memory stages with TMA (no multicast), each stage completing on an mbarrier;
//   - lane 0 of warps 1..NI issue tcgen05.mma (M=128, N=BN, K=16, kind::f16), each into its own
//     TMEM accumulator: one thread's MMAs complete in order at about 130 cycles each whatever N
//     is, so narrow tiles need independent issuers to keep up with the operand stream;
//     every issuer takes its share of each stage's MMAs and releases the stage with
//     tcgen05.commit (the stage's empty barrier counts NI arrivals); the epilogue sums the
//     accumulators in issuer order;
//   - a stage holds GEMM_KPS 64-deep k-blocks of A and W, each operand brought by ONE 3-D TMA
//     box (column-in-block, row, k-block): a TMA request costs ~300 cycles whatever its size, so
//     fewer, larger requests raise a CTA's ingest rate;
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
#include "params.h"

namespace jc {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 256;


// 64-deep k-blocks per pipeline stage: one 3-D TMA box per operand brings all of them.
constexpr int GEMM_KPS = 2;

template <int BN, int STAGES_, int BM_ = GEMM_BM>
struct GemmShape {
    static_assert(BM_ == 128 || BM_ == 64, "128- or 64-row tiles");
    static constexpr int STAGES = STAGES_;
    static constexpr int BM = BM_;
    // Tile rows a warp's 32 TMEM lanes hold: an M = 128 MMA puts row r in lane r; an M = 64 one
    // puts rows 16q..16q + 15 in lanes 32q..32q + 15 (lanes 32q + 16.. hold none).
    static constexpr int RPW = BM_ / 4;
    static constexpr int KPS = GEMM_KPS;
    static constexpr int A_KB = BM_ * GEMM_BK * 2;  // one k-block of A: BM rows x 128 B
    static constexpr int W_KB = BN * GEMM_BK * 2;       // one k-block of W
    static constexpr int A_BYTES = KPS * A_KB;
    static constexpr int B_BYTES = KPS * W_KB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // MMA issuer warps, each with its own accumulator (tcgen05.mma from one thread completes in
    // order at about one 128-row instruction per 130 cycles whatever N is, so narrow tiles need
    // several independent issuers; four measured faster than two for 32- and 64-column tiles).
    static constexpr int NI = BN <= 64 ? 4 : 2;
    static constexpr int ACC_COLS = NI * BN;
    static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                     : ACC_COLS <= 256 ? 256 : 512;
    static constexpr int CH = BN < 64 ? BN : 64;  // epilogue chunk
    static constexpr int G = CH / 4;              // columns per thread per half-chunk group
    static constexpr int NCH = BN / CH;           // chunks per tile
    static constexpr int PER = 2 * G * NCH;       // columns per thread
    // stages | barriers (256 B) | row partial sums (1 KB) | column sums and biases (2 x BN floats)
    // [| cluster split-K receive buffer]
    static constexpr int TAIL_BYTES = 256 + 1024 + 8 * BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + TAIL_BYTES;
    // Cluster split-K over CS CTAs: every CTA receives, from each peer, the partial sums of the
    // columns it owns (GO of each 32-column half of every chunk) for all 128 rows, row-major with
    // rows padded by 4 floats (so a warp's 16-byte accesses of consecutive rows spread over the
    // banks): [CS][NCH][128][RECV_STRIDE] floats (its own rank's slot unused).
    template <int CS>
    static constexpr int RECV_STRIDE = 2 * (2 * (CH / (4 * CS))) + 4;
    template <int CS>
    static constexpr int RECV_BYTES = CS > 1 ? CS * NCH * 128 * RECV_STRIDE<CS> * 4 : 0;
    // Bytes a CTA receives: the partials of its columns from every peer.
    template <int CS>
    static constexpr uint32_t RECV_TX = CS > 1 ? (uint32_t)((CS - 1) * NCH * 128 * 2 * (2 * (CH / (4 * CS))) * 4) : 0;
    static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
};

// G f16 values as G/2 packed half2 words, moved with 16-byte accesses (G % 8 == 0) or 8-byte ones.
template <int G>
__device__ __forceinline__ void load_halves(const __half *src, uint32_t *out) {
    if constexpr (G % 8 == 0) {
#pragma unroll
        for (int j = 0; j < G / 8; j++) {
            const uint4 t = reinterpret_cast<const uint4 *>(src)[j];
            out[4 * j] = t.x; out[4 * j + 1] = t.y; out[4 * j + 2] = t.z; out[4 * j + 3] = t.w;
        }
    } else {
        static_assert(G % 4 == 0, "groups of 4 columns at least");
#pragma unroll
        for (int j = 0; j < G / 4; j++) {
            const uint2 t = reinterpret_cast<const uint2 *>(src)[j];
            out[2 * j] = t.x; out[2 * j + 1] = t.y;
        }
    }
}

template <int G>
__device__ __forceinline__ void store_halves(__half *dst, const uint32_t *in) {
    if constexpr (G % 8 == 0) {
#pragma unroll
        for (int j = 0; j < G / 8; j++)
            reinterpret_cast<uint4 *>(dst)[j] = make_uint4(in[4 * j], in[4 * j + 1], in[4 * j + 2], in[4 * j + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < G / 4; j++)
            reinterpret_cast<uint2 *>(dst)[j] = make_uint2(in[2 * j], in[2 * j + 1]);
    }
}

// Packs G values into G/2 half2 words after adding the residual (already in registers as G/2
// half2 words), and accumulates the statistics of the values as stored (f16), as the next
// LayerNorm sees them.
template <int G, uint32_t EPI>
__device__ __forceinline__ void pack_group(const float *v, const uint32_t *resw, uint32_t *out,
                                           float &s, float &q) {
#pragma unroll
    for (int j = 0; j < G / 2; j++) {
        float lo = v[2 * j], hi = v[2 * j + 1];
        if constexpr ((EPI & JC_EPI_RES) != 0) {
            const float2 r = unpack_half2(resw[j]);
            lo += r.x;
            hi += r.y;
        }
        out[j] = pack_half2(lo, hi);
        if constexpr ((EPI & JC_EPI_STATS) != 0) {
            const float2 f = unpack_half2(out[j]);
            s += f.x + f.y;
            q = fmaf(f.x, f.x, q);
            q = fmaf(f.y, f.y, q);
        }
    }
}

// G f16 values (G/2 words) of tile row `row` at tile-local output column `oc` into the staging
// area of the TMA stores: boxes of BW columns x 128 rows, 16-byte chunk c of a row at chunk
// c ^ (row % 8) (BW 64, 128-byte swizzle) or c ^ ((row / 2) % 4) (BW 32, 64-byte swizzle), the
// layout the tensor map's swizzle mode reads; a warp's 32 rows then spread over all banks.
template <int G, int BW, int BM = GEMM_BM>
__device__ __forceinline__ void stage_halves(uint8_t *stage, uint32_t row, uint32_t oc,
                                             const uint32_t *in) {
    static_assert(G % 8 == 0 && (BW == 64 || BW == 32), "16-byte chunks in 64- or 32-column boxes");
    constexpr uint32_t ROWB = BW * 2;
    uint8_t *box_row = stage + (oc / BW) * (BM * ROWB) + row * ROWB;
    const uint32_t c0 = (oc % BW) / 8;
    const uint32_t sw = BW == 64 ? (row & 7) : ((row >> 1) & 3);
#pragma unroll
    for (int j = 0; j < G / 8; j++)
        *reinterpret_cast<uint4 *>(box_row + (((c0 + j) ^ sw) << 4)) =
            make_uint4(in[4 * j], in[4 * j + 1], in[4 * j + 2], in[4 * j + 3]);
}

// The epilogue of one thread's share of a chunk of 2 * HALF columns starting at global column c0:
// v[0, G) are columns c0 + pair0 + j, v[G, 2G) columns c0 + HALF + pair0 + j (HALF = 32 for the
// 64-column chunks RoPE and GeGLU need: v[j] and v[G + j] are then a RoPE pair (i, i + 32) of one
// head, or a GeGLU input and its gate). cs / bs: the tile's column sums / biases in shared memory
// (tile-local, the tile starting at n0); resw: the residual of those columns (G/2 + G/2 words);
// ropev: (cos, sin) of pairs pair0 .. pair0 + G, two per float4. stage: the TMA-store staging
// area (boxes of BW output columns; tr = the row inside the tile), or nullptr to store directly.
template <int G, int HALF, uint32_t EPI, int BW, int BM = GEMM_BM>
__device__ __forceinline__ void gemm_epilogue_part(const GemmParams &p, float *v, uint32_t r,
                                                   uint32_t tr, uint8_t *stage,
                                                   bool valid, uint32_t n0, uint32_t c0,
                                                   uint32_t pair0, float mean, float rstd,
                                                   const float *cs, const float *bs,
                                                   const uint32_t *resw, const float4 *ropev,
                                                   float &s, float &q) {
    // Staging needs whole 16-byte chunks in 32- or 64-column boxes (every launch the host allows
    // TMA stores for; the other instantiations store directly).
    constexpr bool STAGE_OK = (BW == 32 || BW == 64) && G % 8 == 0;
    const uint32_t la = c0 - n0 + pair0, lb = la + HALF;
    // Column sums and biases from shared memory four at a time (la, lb multiples of 4).
    if constexpr ((EPI & JC_EPI_LN) != 0) {
#pragma unroll
        for (int j = 0; j < G; j += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(cs + la + j);
            const float4 y = *reinterpret_cast<const float4 *>(cs + lb + j);
            v[j] = rstd * (v[j] - mean * x.x);
            v[j + 1] = rstd * (v[j + 1] - mean * x.y);
            v[j + 2] = rstd * (v[j + 2] - mean * x.z);
            v[j + 3] = rstd * (v[j + 3] - mean * x.w);
            v[G + j] = rstd * (v[G + j] - mean * y.x);
            v[G + j + 1] = rstd * (v[G + j + 1] - mean * y.y);
            v[G + j + 2] = rstd * (v[G + j + 2] - mean * y.z);
            v[G + j + 3] = rstd * (v[G + j + 3] - mean * y.w);
        }
    }
    if constexpr ((EPI & JC_EPI_BIAS) != 0) {
#pragma unroll
        for (int j = 0; j < G; j += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(bs + la + j);
            const float4 y = *reinterpret_cast<const float4 *>(bs + lb + j);
            v[j] += x.x; v[j + 1] += x.y; v[j + 2] += x.z; v[j + 3] += x.w;
            v[G + j] += y.x; v[G + j + 1] += y.y; v[G + j + 2] += y.z; v[G + j + 3] += y.w;
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
        static_assert(HALF == 32, "RoPE needs whole 64-column heads");
        // q and k are the first two thirds of a qkv row; the chunk is exactly one head.
        if (valid && c0 < 2 * (p.n / 3)) {
#pragma unroll
            for (int i = 0; i < G / 2; i++) {
                const float4 t = ropev[i];  // (cos, sin) of pairs pair0 + 2i and pair0 + 2i + 1
                float x1 = v[2 * i], x2 = v[2 * i + G];
                v[2 * i] = x1 * t.x - x2 * t.y;
                v[2 * i + G] = x2 * t.x + x1 * t.y;
                x1 = v[2 * i + 1];
                x2 = v[2 * i + 1 + G];
                v[2 * i + 1] = x1 * t.z - x2 * t.w;
                v[2 * i + 1 + G] = x2 * t.z + x1 * t.w;
            }
        }
    }
    if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
        static_assert(HALF == 32, "GeGLU needs 32 input and 32 gate columns per chunk");
        if (valid) {
            // Packed columns [c0, c0 + 32) are GELU inputs of output columns [c0/2, c0/2 + 32),
            // [c0 + 32, c0 + 64) their gates.
            uint32_t out[G / 2];
#pragma unroll
            for (int j = 0; j < G / 2; j++)
                out[j] = pack_half2(gelu_as(v[2 * j]) * v[G + 2 * j],
                                    gelu_as(v[2 * j + 1]) * v[G + 2 * j + 1]);
            if constexpr (STAGE_OK) {
                if (stage) {
                    stage_halves<G, BW, BM>(stage, tr, (c0 - n0) / 2 + pair0, out);
                    return;
                }
            }
            store_halves<G>(p.c + (size_t)r * (p.n / 2) + c0 / 2 + pair0, out);
        }
    } else {
        if (valid) {
            uint32_t oa[G / 2], ob[G / 2];
            pack_group<G, EPI>(v, resw, oa, s, q);
            pack_group<G, EPI>(v + G, resw + G / 2, ob, s, q);
            if constexpr (STAGE_OK) {
                if (stage) {
                    stage_halves<G, BW, BM>(stage, tr, la, oa);
                    stage_halves<G, BW, BM>(stage, tr, lb, ob);
                    return;
                }
            }
            __half *row = p.c + (size_t)r * p.n + n0;
            store_halves<G>(row + la, oa);
            store_halves<G>(row + lb, ob);
        }
    }
}

}  // namespace jc

#include "gemm_tile.cuh"
