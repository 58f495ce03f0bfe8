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
#include "params.h"

namespace jc {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 256;


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

}  // namespace jc

#include "gemm_tile.cuh"
