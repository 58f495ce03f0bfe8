// The reference's per-step GPU forward, restated in CUDA C++ so that it can be timed on the B200
// beside this library (the reference itself is Rust compiled by cuda-oxide, which cannot be
// built here). It is a measurement baseline, not part of the product: nothing in the package
// calls it.
//
// What is restated, and from where:
//   - the GEMM (kernels/src/gemm.rs): BM x 64 tiles on 2*WR warps (WR warp rows x 2 warp columns,
//     each a 16*MI x 32 piece), K in 32-deep steps through two swizzled shared stages filled from
//     registers (the next step's global loads in flight during this step's MMAs), ldmatrix +
//     mma.sync m16n8k16, f32 accumulators in registers (`mainloop` :317-353, `compute` :209-241,
//     `load_regs` / `store_regs` :246-298, `swz` :29);
//   - split-K through a workspace, the last block of a tile summing the partials in split order
//     (`split_reduce` :364-433);
//   - the fused epilogues on the accumulator fragments (kernels/src/main.rs:904-1037): folded
//     LayerNorm, bias, ReLU, GELU, RoPE on q/k rows permuted so a thread holds dims i and i + 32
//     (src/prep.rs:88-101), GeGLU on Wi rows interleaved per n8 fragment (src/prep.rs:67-77),
//     residual + row statistics reduced over the quad and added with `red`;
//   - the zero-clearing of a later GEMM's statistics buffer (kernels/src/main.rs:1074-1084);
//   - attention (kernels/src/main.rs:303-542, kernels/src/attn.rs:20-84): 64 queries of one head
//     per 128-thread block, K and V tiles of 64 keys through swizzled shared memory with the next
//     tile's loads in registers, online softmax in exp2, P.V with V through ldmatrix.trans; window
//     layers visit only reachable key blocks; one key range (the per-step launch);
//   - the launch sequence of src/forward.rs (`launch_layer` :156-165, the head :504-718) and the
//     tile rule of `gemm::choose` (src/gemm.rs:153-180) with this GPU's SM count, plain stream
//     launches (no CUDA graph, no programmatic dependent launch), CUDA events embed -> logits.
// The embedding, head-input and score kernels are this library's own (`edges.cuh`): they restate
// the reference's warp-per-row kernels of the same names and take a few microseconds in total.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../julia-cuda_b200/csrc/edges.cuh"
#include "../../julia-cuda_b200/csrc/model.h"
#include "restated.h"

namespace rs {

using jc::pack_half2;
using jc::unpack_half2;

// ---------------------------------------------------------------------------------------------
// device helpers

constexpr uint32_t BK = 32;

// Element offset of (row, 16-byte chunk) in a swizzled [rows][32] f16 tile (gemm.rs:29).
__device__ __forceinline__ uint32_t swz32(uint32_t row, uint32_t chunk) {
    return row * BK + ((chunk ^ ((row >> 1) & 3)) << 3);
}

// Element offset of (row, 16-byte chunk) in a swizzled [rows][64] f16 tile (attn.rs:26-28).
__device__ __forceinline__ uint32_t swz64(uint32_t row, uint32_t chunk) {
    return row * 64 + ((chunk ^ (row & 7)) << 3);
}

__device__ __forceinline__ uint32_t saddr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// c += a . b for one 16 x 8 x 16 step.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void red_add(float *p, float x) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(x) : "memory");
}

// ---------------------------------------------------------------------------------------------
// GEMM

struct GemmP {
    const __half *a, *w;
    __half *c;
    const __half *res;
    float *ws;
    uint32_t *counters;
    const float *stats_in, *colsum;
    float *stats_out, *zero;
    uint32_t zero_len, m, n, k;
    float eps;
    const float *rope, *bias;
};

// The next K step's chunks into registers: A chunks tid + 64 WR h (h < MI; rows past m zero),
// then 4 / WR W chunks (gemm.rs:246-278).
template <int MI, int WR>
__device__ __forceinline__ void load_regs(const GemmP &g, uint32_t bx, uint32_t by, uint32_t k0, uint4 (&v)[MI + 2]) {
    constexpr uint32_t NT = 64 * WR, BM = 16 * MI * WR;
    const uint32_t tid = threadIdx.x;
#pragma unroll
    for (int h = 0; h < MI; h++) {
        const uint32_t ch = tid + h * NT, row = ch >> 2, col = k0 + (ch & 3) * 8;
        const uint32_t ar = by * BM + row;
        v[h] = ar < g.m ? *reinterpret_cast<const uint4 *>(g.a + (size_t)ar * g.k + col) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int h = 0; h < 4 / WR; h++) {
        const uint32_t ch = tid + h * NT, row = ch >> 2, col = k0 + (ch & 3) * 8;
        v[MI + h] = *reinterpret_cast<const uint4 *>(g.w + (size_t)(bx * 64 + row) * g.k + col);
    }
}

template <int MI, int WR>
__device__ __forceinline__ void store_regs(const uint4 (&v)[MI + 2], uint16_t *a_s, uint16_t *w_s) {
    constexpr uint32_t NT = 64 * WR;
    const uint32_t tid = threadIdx.x;
#pragma unroll
    for (int h = 0; h < MI; h++) {
        const uint32_t ch = tid + h * NT;
        *reinterpret_cast<uint4 *>(a_s + swz32(ch >> 2, ch & 3)) = v[h];
    }
#pragma unroll
    for (int h = 0; h < 4 / WR; h++) {
        const uint32_t ch = tid + h * NT;
        *reinterpret_cast<uint4 *>(w_s + swz32(ch >> 2, ch & 3)) = v[MI + h];
    }
}

// One 32-deep step of this warp's 16 MI x 32 piece (gemm.rs:209-241).
template <int MI>
__device__ __forceinline__ void compute(float (&acc)[MI][4][4], const uint16_t *a_s, const uint16_t *w_s) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t wm = (warp >> 1) * 16 * MI, wn = (warp & 1) * 32;
#pragma unroll
    for (uint32_t ks = 0; ks < 2; ks++) {
        const uint32_t nrow = (lane & 7) + ((lane >> 4) << 3), kc = ks * 2 + ((lane >> 3) & 1);
        uint32_t b[2][4];
        ldsm_x4(saddr(w_s + swz32(wn + nrow, kc)), b[0]);
        ldsm_x4(saddr(w_s + swz32(wn + 16 + nrow, kc)), b[1]);
#pragma unroll
        for (int i = 0; i < MI; i++) {
            uint32_t a[4];
            ldsm_x4(saddr(a_s + swz32(wm + i * 16 + (lane & 15), ks * 2 + (lane >> 4))), a);
#pragma unroll
            for (int j = 0; j < 4; j++) mma16816(acc[i][j], a, b[j >> 1][(j & 1) * 2], b[j >> 1][(j & 1) * 2 + 1]);
        }
    }
}

template <int MI, int WR, uint32_t EPI>
__global__ void __launch_bounds__(64 * WR) gemm_kernel(const GemmP g) {
    constexpr uint32_t NT = 64 * WR, BM = 16 * MI * WR;
    __shared__ __align__(128) uint16_t smem[2 * (BM * BK + 64 * BK)];
    __shared__ uint32_t last_s;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bx = blockIdx.x, by = blockIdx.y, z = blockIdx.z, splits = gridDim.z;

    // The statistics buffer a later GEMM adds into, cleared on the way.
    const uint32_t blocks = gridDim.x * gridDim.y * gridDim.z;
    const uint32_t flat = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    for (uint32_t i = flat * NT + tid; i < g.zero_len; i += blocks * NT) g.zero[i] = 0.0f;

    float acc[MI][4][4];
#pragma unroll
    for (int i = 0; i < MI; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[i][j][e] = 0.0f;

    const uint32_t nk = g.k / BK, kt0 = z * nk / splits, kt1 = (z + 1) * nk / splits;
    uint16_t *a_s = smem, *w_s = smem + 2 * BM * BK;
    uint4 v[MI + 2];
    load_regs<MI, WR>(g, bx, by, kt0 * BK, v);
    store_regs<MI, WR>(v, a_s, w_s);
    __syncthreads();
    for (uint32_t kt = kt0; kt < kt1; kt++) {
        if (kt + 1 < kt1) load_regs<MI, WR>(g, bx, by, (kt + 1) * BK, v);
        const uint32_t cur = (kt - kt0) & 1;
        compute<MI>(acc, a_s + cur * BM * BK, w_s + cur * 64 * BK);
        if (kt + 1 < kt1) store_regs<MI, WR>(v, a_s + (1 - cur) * BM * BK, w_s + (1 - cur) * 64 * BK);
        __syncthreads();
    }

    if (splits > 1) {
        // Every split stores its partial ([fragment][thread] float4s); the last to arrive sums
        // them all in split order and runs the epilogue.
        const uint32_t tile = by * gridDim.x + bx;
        float4 *mine = reinterpret_cast<float4 *>(g.ws + (size_t)(tile * splits + z) * 1024 * MI * WR);
#pragma unroll
        for (int i = 0; i < MI; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
                mine[(i * 4 + j) * NT + tid] = make_float4(acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3]);
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t old = atomicAdd(g.counters + tile, 1u);
            const bool is_last = old == splits - 1;
            if (is_last) g.counters[tile] = 0;
            last_s = is_last ? 1u : 0u;
        }
        __syncthreads();
        if (!last_s) return;
        __threadfence();
#pragma unroll
        for (int i = 0; i < MI; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[i][j][e] = 0.0f;
        for (uint32_t s = 0; s < splits; s++) {
            const float4 *p = reinterpret_cast<const float4 *>(g.ws + (size_t)(tile * splits + s) * 1024 * MI * WR);
#pragma unroll
            for (int i = 0; i < MI; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 t = __ldcg(p + (i * 4 + j) * NT + tid);
                    acc[i][j][0] += t.x;
                    acc[i][j][1] += t.y;
                    acc[i][j][2] += t.z;
                    acc[i][j][3] += t.w;
                }
        }
    }

    // Epilogue on the fragments: thread holds rows r0 + 16 i + 8 h, columns cw + 8 j (+0, +1).
    const uint32_t r0 = by * BM + (warp >> 1) * 16 * MI + (lane >> 2);
    const uint32_t cw = bx * 64 + (warp & 1) * 32 + (lane & 3) * 2;
#pragma unroll
    for (int i = 0; i < MI; i++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t r = r0 + i * 16 + h * 8;
            const bool ok = r < g.m;
            float2 v2[4];
#pragma unroll
            for (int j = 0; j < 4; j++) v2[j] = make_float2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
            if constexpr ((EPI & JC_EPI_LN) != 0) {
                if (ok) {
                    const float s = g.stats_in[2 * r], q = g.stats_in[2 * r + 1];
                    const float mean = s / (float)g.k, var = q / (float)g.k - mean * mean;
                    const float rstd = rsqrtf((var > 0.0f ? var : 0.0f) + g.eps);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint32_t col = cw + j * 8;
                        v2[j] = make_float2(rstd * (v2[j].x - mean * g.colsum[col]),
                                            rstd * (v2[j].y - mean * g.colsum[col + 1]));
                    }
                }
            }
            if constexpr ((EPI & JC_EPI_BIAS) != 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t col = cw + j * 8;
                    v2[j].x += g.bias[col];
                    v2[j].y += g.bias[col + 1];
                }
            }
            if constexpr ((EPI & JC_EPI_RELU) != 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) v2[j] = make_float2(fmaxf(v2[j].x, 0.0f), fmaxf(v2[j].y, 0.0f));
            }
            if constexpr ((EPI & JC_EPI_GELU) != 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) v2[j] = make_float2(jc::gelu_as(v2[j].x), jc::gelu_as(v2[j].y));
            }
            if constexpr ((EPI & JC_EPI_ROPE) != 0) {
                if (ok) {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint32_t col = cw + j * 8;
                        if (col < 2 * (g.n / 3)) {
                            // Permuted rows: the pair (2p, 2p + 1) is dims p and p + 32.
                            const uint32_t pair = (col % 64) / 2;
                            const float cs = g.rope[((size_t)r * 32 + pair) * 2], sn = g.rope[((size_t)r * 32 + pair) * 2 + 1];
                            const float x1 = v2[j].x, x2 = v2[j].y;
                            v2[j] = make_float2(x1 * cs - x2 * sn, x2 * cs + x1 * sn);
                        }
                    }
                }
            }
            if constexpr ((EPI & JC_EPI_GEGLU) != 0) {
                // Fragments 2q and 2q + 1 are the GELU inputs and gates of the same 8 columns.
                const uint32_t c0 = bx * 32 + (warp & 1) * 16 + (lane & 3) * 2;
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    if (ok) {
                        const float2 x = v2[2 * q], gt = v2[2 * q + 1];
                        *reinterpret_cast<uint32_t *>(g.c + (size_t)r * (g.n / 2) + c0 + q * 8) =
                            pack_half2(jc::gelu_as(x.x) * gt.x, jc::gelu_as(x.y) * gt.y);
                    }
                }
            } else {
                float s = 0.0f, s2 = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (ok) {
                        const size_t idx = (size_t)r * g.n + cw + j * 8;
                        float lo = v2[j].x, hi = v2[j].y;
                        if constexpr ((EPI & JC_EPI_RES) != 0) {
                            const float2 x = unpack_half2(*reinterpret_cast<const uint32_t *>(g.res + idx));
                            lo += x.x;
                            hi += x.y;
                        }
                        const uint32_t packed = pack_half2(lo, hi);
                        *reinterpret_cast<uint32_t *>(g.c + idx) = packed;
                        if constexpr ((EPI & JC_EPI_STATS) != 0) {
                            const float2 x = unpack_half2(packed);
                            s += x.x + x.y;
                            s2 += x.x * x.x + x.y * x.y;
                        }
                    }
                }
                if constexpr ((EPI & JC_EPI_STATS) != 0) {
                    // The quad of lanes holding a row's 32 columns of this warp.
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
                    if (ok && (lane & 3) == 0) {
                        red_add(g.stats_out + 2 * (size_t)r, s);
                        red_add(g.stats_out + 2 * (size_t)r + 1, s2);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// attention

// Thread t's 4 chunks (16 bytes; chunk c = t + 128 i is row c / 8, chunk c % 8) of one head's 64
// rows from row0 of third `third` (0 q, 1 k, 2 v); rows past n zero (attn.rs:51-70).
__device__ __forceinline__ void load_tile(const __half *qkv, uint32_t n, uint32_t d, uint32_t row0,
                                          uint32_t head, uint32_t third, uint4 (&v)[4]) {
#pragma unroll
    for (uint32_t i = 0; i < 4; i++) {
        const uint32_t c = threadIdx.x + 128 * i, row = c >> 3, ch = c & 7, r = row0 + row;
        v[i] = r < n ? *reinterpret_cast<const uint4 *>(qkv + (size_t)r * 3 * d + third * d + head * 64 + ch * 8)
                     : make_uint4(0, 0, 0, 0);
    }
}

__device__ __forceinline__ void store_tile(uint16_t *tile, const uint4 (&v)[4]) {
#pragma unroll
    for (uint32_t i = 0; i < 4; i++) {
        const uint32_t c = threadIdx.x + 128 * i;
        *reinterpret_cast<uint4 *>(tile + swz64(c >> 3, c & 7)) = v[i];
    }
}

__global__ void __launch_bounds__(128) attention_kernel(const __half *qkv, __half *o, uint32_t n,
                                                        uint32_t window, uint32_t d) {
    __shared__ __align__(128) uint16_t qs[64 * 64], ks[64 * 64], vs[64 * 64];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t q0 = blockIdx.x * 64, head = blockIdx.y;
    const uint32_t nb = (n + 63) / 64;
    uint32_t kb0 = 0, kb1 = nb;
    if (window != 0) {
        kb0 = (q0 > window ? q0 - window : 0) / 64;
        kb1 = min(q0 + 63 + window, n - 1) / 64 + 1;
    }
    uint32_t qf[4][4];
    uint4 kn[4], vn[4];
    if (kb0 < kb1) {
        uint4 q[4];
        load_tile(qkv, n, d, q0, head, 0, q);
        load_tile(qkv, n, d, kb0 * 64, head, 1, kn);
        load_tile(qkv, n, d, kb0 * 64, head, 2, vn);
        store_tile(qs, q);
        __syncthreads();
#pragma unroll
        for (uint32_t kk = 0; kk < 4; kk++) ldsm_x4(saddr(qs + swz64(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))), qf[kk]);
    }
    const float scale = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
    const uint32_t gq = lane >> 2, t = lane & 3;
    const uint32_t qrow[2] = {q0 + warp * 16 + gq, q0 + warp * 16 + gq + 8};
    float mx[2] = {-INFINITY, -INFINITY}, sum[2] = {0.0f, 0.0f};
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[j][e] = 0.0f;

    for (uint32_t kb = kb0; kb < kb1; kb++) {
        const uint32_t k0 = kb * 64;
        store_tile(ks, kn);
        store_tile(vs, vn);
        __syncthreads();
        if (kb + 1 < kb1) {
            load_tile(qkv, n, d, k0 + 64, head, 1, kn);
            load_tile(qkv, n, d, k0 + 64, head, 2, vn);
        }
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) s[j][e] = 0.0f;
        const uint32_t nrow = (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; kk++) {
            const uint32_t kc = kk * 2 + ((lane >> 3) & 1);
#pragma unroll
            for (uint32_t jp = 0; jp < 4; jp++) {
                uint32_t b[4];
                ldsm_x4(saddr(ks + swz64(16 * jp + nrow, kc)), b);
                mma16816(s[2 * jp], qf[kk], b[0], b[1]);
                mma16816(s[2 * jp + 1], qf[kk], b[2], b[3]);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float m = -INFINITY;
#pragma unroll
            for (uint32_t jt = 0; jt < 8; jt++)
#pragma unroll
                for (uint32_t e = 0; e < 2; e++) {
                    const uint32_t key = k0 + 8 * jt + 2 * t + e, q = qrow[h];
                    const bool near = window == 0 || (q > key ? q - key : key - q) <= window;
                    float &x = s[jt][2 * h + e];
                    x = key < n && near ? x * scale : -INFINITY;
                    m = fmaxf(m, x);
                }
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            const float m_new = fmaxf(m, mx[h]);
            const float base = m_new == -INFINITY ? 0.0f : m_new;
            const float alpha = ex2(mx[h] - base);
            mx[h] = m_new;
            float rsum = 0.0f;
#pragma unroll
            for (int jt = 0; jt < 8; jt++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float p = ex2(s[jt][2 * h + e] - base);
                    s[jt][2 * h + e] = p;
                    rsum += p;
                }
                acc[jt][2 * h] *= alpha;
                acc[jt][2 * h + 1] *= alpha;
            }
            sum[h] = sum[h] * alpha + rsum;
        }
#pragma unroll
        for (uint32_t kk = 0; kk < 4; kk++) {
            const uint32_t a[4] = {pack_half2(s[2 * kk][0], s[2 * kk][1]), pack_half2(s[2 * kk][2], s[2 * kk][3]),
                                   pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                                   pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
            for (uint32_t dp = 0; dp < 4; dp++) {
                uint32_t vv[4];
                ldsm_x4_trans(saddr(vs + swz64(16 * kk + (lane & 15), 2 * dp + (lane >> 4))), vv);
                mma16816(acc[2 * dp], a, vv[0], vv[1]);
                mma16816(acc[2 * dp + 1], a, vv[2], vv[3]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float l = sum[h];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        if (qrow[h] < n) {
#pragma unroll
            for (uint32_t jt = 0; jt < 8; jt++) {
                const uint32_t col = head * 64 + 8 * jt + 2 * t;
                *reinterpret_cast<uint32_t *>(o + (size_t)qrow[h] * d + col) =
                    pack_half2(acc[jt][2 * h] * inv, acc[jt][2 * h + 1] * inv);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// launches

// gemm::choose (src/gemm.rs:153-180): the tile height from m (32 up to 200 rows, 64 up to 400,
// else 128 on 8 warps), split-K 4 while the tiles fill at most half the SMs, at least 3 K steps
// a split.
struct Plan {
    int shape;
    uint32_t bm, splits;
};

static Plan choose(uint32_t m, uint32_t n, uint32_t k, int sms) {
    Plan p;
    p.shape = m <= 200 ? 0 : (m <= 400 ? 1 : 2);
    p.bm = p.shape == 0 ? 32 : (p.shape == 1 ? 64 : 128);
    const uint32_t tiles = (n / 64) * ((m + p.bm - 1) / p.bm);
    p.splits = 2 * tiles > (uint32_t)sms ? 1 : 4;
    p.splits = std::min(p.splits, std::max(k / 32 / 3, 1u));
    return p;
}

template <uint32_t EPI>
static void launch_gemm(const GemmP &g, int sms, cudaStream_t stream) {
    const Plan p = choose(g.m, g.n, g.k, sms);
    const dim3 grid(g.n / 64, (g.m + p.bm - 1) / p.bm, p.splits);
    if (p.shape == 0)
        gemm_kernel<1, 2, EPI><<<grid, 128, 0, stream>>>(g);
    else if (p.shape == 1)
        gemm_kernel<2, 2, EPI><<<grid, 128, 0, stream>>>(g);
    else
        gemm_kernel<2, 4, EPI><<<grid, 256, 0, stream>>>(g);
}

static bool launch_gemm_epi(uint32_t epi, const GemmP &g, int sms, cudaStream_t stream) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    switch (epi) {
        case JC_EPI_ROPE: launch_gemm<JC_EPI_ROPE>(g, sms, stream); return true;
        case JC_EPI_LN | JC_EPI_ROPE: launch_gemm<JC_EPI_LN | JC_EPI_ROPE>(g, sms, stream); return true;
        case JC_EPI_LN | JC_EPI_GEGLU: launch_gemm<JC_EPI_LN | JC_EPI_GEGLU>(g, sms, stream); return true;
        case RS: launch_gemm<RS>(g, sms, stream); return true;
        case JC_EPI_BIAS | RS: launch_gemm<JC_EPI_BIAS | RS>(g, sms, stream); return true;
        case LB: launch_gemm<LB>(g, sms, stream); return true;
        case LB | JC_EPI_RELU: launch_gemm<LB | JC_EPI_RELU>(g, sms, stream); return true;
        case LB | JC_EPI_GELU: launch_gemm<LB | JC_EPI_GELU>(g, sms, stream); return true;
        default: return false;
    }
}

// ---------------------------------------------------------------------------------------------
// host: weights in the reference's layouts, buffers, the launch sequence

// Wqkv rows for the fragment RoPE epilogue: in each q and k head, packed rows 2i and 2i + 1 are
// dims i and i + 32 (src/prep.rs:88-101); v rows stay in order.
static uint32_t rope_src_row(uint32_t p, uint32_t n) {
    if (p >= 2 * n / 3) return p;
    const uint32_t head = p / 64, i = p % 64;
    return head * 64 + i / 2 + (i % 2) * 32;
}

// Wi rows for the fragment GeGLU epilogue: packed row p = 64t + 32h + 16q + 8s + e is source row
// 32t + 16h + 8q + e (+ intermediate for the gate, s = 1) (src/prep.rs:67-77).
static uint32_t geglu_src_row(uint32_t p, uint32_t n) {
    const uint32_t t = p / 64, h = (p % 64) / 32, q = (p % 32) / 16, s = (p % 16) / 8, e = p % 8;
    return t * 32 + h * 16 + q * 8 + e + (s ? n / 2 : 0);
}

struct Linear {
    __half *w = nullptr;
    float *colsum = nullptr, *bias = nullptr;
};

struct Restated {
    jc_model_config c{};
    int sms = 0;
    size_t max_len = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<void *> allocs;
    // weights
    __half *tok_emb = nullptr;
    float *emb_norm = nullptr, *final_norm = nullptr, *type_emb = nullptr, *rope_g = nullptr, *rope_l = nullptr;
    std::vector<Linear> qkv, wo, wi, wo_mlp, h_in, h_out, h_l1, h_l2;
    Linear s_lin1;
    __half *s_lin2 = nullptr;
    float s_lin2_b = 0.0f;
    // encoder buffers
    __half *x = nullptr, *qkvb = nullptr, *o = nullptr, *m = nullptr;
    float *stats_attn = nullptr, *stats_mlp = nullptr;
    // head buffers (the reference's GpuHead has its own)
    __half *hx = nullptr, *hqkv = nullptr, *ho = nullptr, *hf = nullptr, *hy = nullptr;
    float *stats_a = nullptr, *stats_b = nullptr, *logits = nullptr;
    uint32_t *ids = nullptr, *markers = nullptr;
    // split-K scratch
    float *ws = nullptr;
    uint32_t *counters = nullptr;
    std::string err;

    template <typename T>
    T *dev(size_t count) {
        void *p = nullptr;
        if (cudaMalloc(&p, count * sizeof(T) + 16) != cudaSuccess) return nullptr;
        allocs.push_back(p);
        cudaMemset(p, 0, count * sizeof(T) + 16);
        return static_cast<T *>(p);
    }
    template <typename T>
    T *upload(const std::vector<T> &h) {
        T *p = dev<T>(h.size());
        if (p) cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
        return p;
    }

    ~Restated() {
        for (void *p : allocs) cudaFree(p);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (stream) cudaStreamDestroy(stream);
    }

    Linear plain(const float *w, uint32_t out, uint32_t k, const float *bias, uint32_t (*perm)(uint32_t, uint32_t)) {
        std::vector<uint16_t> h((size_t)out * k);
        for (uint32_t p = 0; p < out; p++) {
            const uint32_t src = perm ? perm(p, out) : p;
            for (uint32_t j = 0; j < k; j++) h[(size_t)p * k + j] = jc::f16_bits(w[(size_t)src * k + j]);
        }
        Linear L;
        L.w = reinterpret_cast<__half *>(upload(h));
        if (bias) L.bias = upload(std::vector<float>(bias, bias + out));
        return L;
    }

    // LayerNorm folded into the linear (colsum from the rounded weights; with a LayerNorm bias,
    // b + W.beta), then the rows reordered by perm.
    Linear folded(const float *w, const float *gamma, const float *beta, const float *b, uint32_t out,
                  uint32_t k, uint32_t (*perm)(uint32_t, uint32_t)) {
        std::vector<uint16_t> w16((size_t)out * k), pw((size_t)out * k);
        std::vector<float> cs(out), pcs(out), bias(out), pb(out);
        if (beta)
            jc::fold_layernorm_bias(w, gamma, beta, b, out, k, w16.data(), cs.data(), bias.data());
        else
            jc::fold_layernorm(w, gamma, out, k, w16.data(), cs.data());
        for (uint32_t p = 0; p < out; p++) {
            const uint32_t src = perm ? perm(p, out) : p;
            std::memcpy(&pw[(size_t)p * k], &w16[(size_t)src * k], k * 2);
            pcs[p] = cs[src];
            pb[p] = bias[src];
        }
        Linear L;
        L.w = reinterpret_cast<__half *>(upload(pw));
        L.colsum = upload(pcs);
        if (beta) L.bias = upload(pb);
        return L;
    }

    bool load(const jc_model_config &cfg, const float *raw, size_t max_length, int device) {
        c = cfg;
        std::string why;
        if (!jc::check_config(c, &why)) return fail("config: " + why);
        if (c.d_model != 768 && c.d_model != 384) return fail("the restated path covers widths 384 and 768");
        if (cudaSetDevice(device) != cudaSuccess) return fail("cudaSetDevice failed");
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        max_len = max_length ? max_length : (size_t)c.max_positions;
        if (max_len > (size_t)c.max_positions) return fail("max_length above max_positions");
        if (cudaStreamCreate(&stream) != cudaSuccess || cudaEventCreate(&ev0) != cudaSuccess ||
            cudaEventCreate(&ev1) != cudaSuccess)
            return fail("stream / event creation failed");
        const jc::RawLayout L = jc::raw_layout(c);
        const uint32_t D = c.d_model, I = c.inter, F = c.head_ff, S = c.scorer_hidden;
        auto at = [&](const jc::Span &s) { return raw + s.off; };
        {
            std::vector<uint16_t> t(L.tok_emb.len);
            for (size_t i = 0; i < t.size(); i++) t[i] = jc::f16_bits(raw[L.tok_emb.off + i]);
            tok_emb = reinterpret_cast<__half *>(upload(t));
        }
        emb_norm = upload(std::vector<float>(at(L.emb_norm), at(L.emb_norm) + D));
        final_norm = upload(std::vector<float>(at(L.final_norm), at(L.final_norm) + D));
        type_emb = upload(std::vector<float>(at(L.type_emb), at(L.type_emb) + L.type_emb.len));
        std::vector<float> tab((size_t)max_len * 64);
        jc::rope_table(c.theta_global, (uint32_t)max_len, tab.data());
        rope_g = upload(tab);
        jc::rope_table(c.theta_local, (uint32_t)max_len, tab.data());
        rope_l = upload(tab);
        for (int l = 0; l < c.n_layers; l++) {
            if (l == 0)
                qkv.push_back(plain(at(L.wqkv[l]), 3 * D, D, nullptr, rope_src_row));
            else
                qkv.push_back(folded(at(L.wqkv[l]), at(L.attn_norm[l]), nullptr, nullptr, 3 * D, D, rope_src_row));
            wo.push_back(plain(at(L.wo[l]), D, D, nullptr, nullptr));
            wi.push_back(folded(at(L.wi[l]), at(L.mlp_norm[l]), nullptr, nullptr, 2 * I, D, geglu_src_row));
            wo_mlp.push_back(plain(at(L.wo_mlp[l]), D, I, nullptr, nullptr));
        }
        for (int l = 0; l < c.n_head_layers; l++) {
            h_in.push_back(folded(at(L.h_in_w[l]), at(L.h_norm1_w[l]), at(L.h_norm1_b[l]), at(L.h_in_b[l]), 3 * D, D, nullptr));
            h_out.push_back(plain(at(L.h_out_w[l]), D, D, at(L.h_out_b[l]), nullptr));
            h_l1.push_back(folded(at(L.h_l1_w[l]), at(L.h_norm2_w[l]), at(L.h_norm2_b[l]), at(L.h_l1_b[l]), F, D, nullptr));
            h_l2.push_back(plain(at(L.h_l2_w[l]), D, F, at(L.h_l2_b[l]), nullptr));
        }
        s_lin1 = folded(at(L.s_lin1_w), at(L.s_norm_w), at(L.s_norm_b), at(L.s_lin1_b), S, D, nullptr);
        s_lin2 = plain(at(L.s_lin2_w), 1, S, nullptr, nullptr).w;
        s_lin2_b = raw[L.s_lin2_b.off];
        const size_t n = max_len;
        x = dev<__half>(n * D);
        qkvb = dev<__half>(n * 3 * D);
        o = dev<__half>(n * D);
        m = dev<__half>(n * I);
        stats_attn = dev<float>(2 * n);
        stats_mlp = dev<float>(2 * n);
        hx = dev<__half>(n * D);
        hqkv = dev<__half>(n * 3 * D);
        ho = dev<__half>(n * D);
        hf = dev<__half>(n * F);
        hy = dev<__half>(n * S);
        stats_a = dev<float>(2 * n);
        stats_b = dev<float>(2 * n);
        logits = dev<float>(n);
        ids = dev<uint32_t>(n);
        markers = dev<uint32_t>(n);
        // Split-K scratch as src/gemm.rs:201-216, for the widest GEMM of this model.
        const size_t max_n = std::max(std::max<size_t>(3 * D, 2 * I), (size_t)F);
        ws = dev<float>(4 * (n + 127) * max_n);
        counters = dev<uint32_t>((max_n / 64) * ((n + 31) / 32));
        if (!ws || !counters || !logits) return fail("device allocation failed");
        if (cudaDeviceSynchronize() != cudaSuccess) return fail("upload failed");
        return true;
    }

    bool fail(const std::string &s) {
        err = s;
        return false;
    }

    template <uint32_t EPI>
    void gemm(const __half *a, const Linear &w, uint32_t mm, uint32_t nn, uint32_t kk, __half *cc,
              const __half *res, const float *stats_in, float *stats_out, float *zero, uint32_t zero_len,
              float eps, const float *rope) {
        const GemmP g{a, w.w, cc, res, ws, counters, stats_in, w.colsum, stats_out, zero, zero_len, mm, nn, kk, eps, rope, w.bias};
        launch_gemm<EPI>(g, sms, stream);
    }

    void attention(const __half *q, __half *out, uint32_t n, uint32_t window) {
        attention_kernel<<<dim3((n + 63) / 64, c.n_heads), 128, 0, stream>>>(q, out, n, window, c.d_model);
    }

    template <int D>
    void forward(uint32_t n, uint32_t nm, uint32_t qtype) {
        constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
        const uint32_t I = c.inter, F = c.head_ff, S = c.scorer_hidden;
        const float eps = c.norm_eps, heps = c.head_eps;
        jc::embed_kernel<D><<<(n + 3) / 4, 128, 0, stream>>>(ids, n, tok_emb, emb_norm, eps, x, nullptr);
        for (int l = 0; l < c.n_layers; l++) {
            const bool global = l % c.global_every == 0;
            const float *rope = global ? rope_g : rope_l;
            if (l == 0)
                gemm<JC_EPI_ROPE>(x, qkv[l], n, 3 * D, D, qkvb, nullptr, nullptr, nullptr, stats_attn, 2 * n, eps, rope);
            else
                gemm<JC_EPI_LN | JC_EPI_ROPE>(x, qkv[l], n, 3 * D, D, qkvb, nullptr, stats_mlp, nullptr, stats_attn, 2 * n, eps, rope);
            attention(qkvb, o, n, global ? 0u : (uint32_t)c.window);
            gemm<RS>(o, wo[l], n, D, D, x, x, nullptr, stats_attn, nullptr, 0, eps, nullptr);
            gemm<JC_EPI_LN | JC_EPI_GEGLU>(x, wi[l], n, 2 * I, D, m, nullptr, stats_attn, nullptr, stats_mlp, 2 * n, eps, nullptr);
            gemm<RS>(m, wo_mlp[l], n, D, I, x, x, nullptr, stats_mlp, nullptr, 0, eps, nullptr);
        }
        jc::norm_add_kernel<D><<<(n + 3) / 4, 128, 0, stream>>>(x, n, final_norm, type_emb + (size_t)qtype * D, eps, hx, stats_a);
        for (int l = 0; l < c.n_head_layers; l++) {
            gemm<LB>(hx, h_in[l], n, 3 * D, D, hqkv, nullptr, stats_a, nullptr, stats_b, 2 * n, heps, nullptr);
            attention(hqkv, ho, n, 0);
            gemm<JC_EPI_BIAS | RS>(ho, h_out[l], n, D, D, hx, hx, nullptr, stats_b, nullptr, 0, heps, nullptr);
            gemm<LB | JC_EPI_RELU>(hx, h_l1[l], n, F, D, hf, nullptr, stats_b, nullptr, stats_a, 2 * n, heps, nullptr);
            gemm<JC_EPI_BIAS | RS>(hf, h_l2[l], n, D, F, hx, hx, nullptr, stats_a, nullptr, 0, heps, nullptr);
        }
        // The scorer on every row (src/forward.rs:662-718), then the marker rows' logits.
        gemm<LB | JC_EPI_GELU>(hx, s_lin1, n, S, D, hy, nullptr, stats_a, nullptr, nullptr, 0, heps, nullptr);
        jc::score_kernel<<<(nm + 3) / 4, 128, 0, stream>>>(hy, S, s_lin2, s_lin2_b, markers, nm, logits);
    }

    int run(const uint32_t *h_ids, size_t n, const uint32_t *h_markers, size_t nm, uint32_t qtype,
            float *h_logits, float *gpu_ms) {
        if (n < 1 || n > max_len) return fail("sequence length out of range"), -1;
        if (nm < 1 || nm > n) return fail("marker count out of range"), -1;
        for (size_t i = 0; i < nm; i++)
            if (h_markers[i] >= n) return fail("marker past the sequence"), -1;
        for (size_t i = 0; i < n; i++)
            if (h_ids[i] >= (uint32_t)c.vocab) return fail("token id past the vocabulary"), -1;
        if (qtype >= (uint32_t)c.n_qtypes) return fail("no such question type"), -1;
        cudaMemcpyAsync(ids, h_ids, n * 4, cudaMemcpyHostToDevice, stream);
        cudaMemcpyAsync(markers, h_markers, nm * 4, cudaMemcpyHostToDevice, stream);
        cudaEventRecord(ev0, stream);
        if (c.d_model == 768)
            forward<768>((uint32_t)n, (uint32_t)nm, qtype);
        else
            forward<384>((uint32_t)n, (uint32_t)nm, qtype);
        cudaEventRecord(ev1, stream);
        cudaMemcpyAsync(h_logits, logits, nm * 4, cudaMemcpyDeviceToHost, stream);
        const cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return fail(std::string("forward failed: ") + cudaGetErrorString(e)), -1;
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev0, ev1);
        if (gpu_ms) *gpu_ms = ms;
        for (size_t i = 0; i < nm; i++)
            if (!std::isfinite(h_logits[i])) return fail("non-finite logits"), -1;
        return 0;
    }
};

static void put_err(const std::string &s, char *err, size_t len) {
    if (!err || !len) return;
    const size_t k = std::min(len - 1, s.size());
    std::memcpy(err, s.data(), k);
    err[k] = 0;
}

}  // namespace rs

extern "C" {

void *jc_restated_load(const jc_model_config *cfg, const float *raw, size_t raw_len, size_t max_length,
                       int device, char *err, size_t err_len) {
    if (!cfg || !raw || raw_len != jc::raw_layout(*cfg).total) {
        rs::put_err("restated: missing config or raw weights of the wrong size", err, err_len);
        return nullptr;
    }
    auto *r = new rs::Restated();
    if (!r->load(*cfg, raw, max_length, device)) {
        rs::put_err("restated: " + r->err, err, err_len);
        delete r;
        return nullptr;
    }
    return r;
}

int jc_restated_run(void *h, const uint32_t *ids, size_t n, const uint32_t *markers, size_t n_markers,
                    uint32_t qtype, float *logits, float *gpu_ms, char *err, size_t err_len) {
    auto *r = static_cast<rs::Restated *>(h);
    if (!r || !ids || !markers || !logits) {
        rs::put_err("restated: null argument", err, err_len);
        return -1;
    }
    if (r->run(ids, n, markers, n_markers, qtype, logits, gpu_ms) != 0) {
        rs::put_err("restated: " + r->err, err, err_len);
        return -1;
    }
    return 0;
}

void jc_restated_free(void *h) { delete static_cast<rs::Restated *>(h); }

size_t jc_restated_gemm_ws_floats(uint32_t m, uint32_t n, uint32_t k, int sms) {
    const rs::Plan p = rs::choose(m, n, k, sms);
    return p.splits > 1 ? (size_t)(n / 64) * ((m + p.bm - 1) / p.bm) * p.splits * p.bm * 64 : 0;
}

size_t jc_restated_gemm_counters(uint32_t m, uint32_t n, uint32_t k, int sms) {
    const rs::Plan p = rs::choose(m, n, k, sms);
    return p.splits > 1 ? (size_t)(n / 64) * ((m + p.bm - 1) / p.bm) : 0;
}

int jc_restated_gemm(uint32_t epi, const void *a, const void *w, void *c, const void *res, float *ws,
                     uint32_t *counters, const float *stats_in, const float *colsum, float *stats_out,
                     float *zero, uint32_t zero_len, uint32_t m, uint32_t n, uint32_t k, float eps,
                     const float *rope, const float *bias, int sms, void *stream) {
    if (m < 1 || n % 64 || k % 32 || k < 32 || !a || !w || !c || sms < 1) return -1;
    if (jc_restated_gemm_ws_floats(m, n, k, sms) && (!ws || !counters)) return -1;
    const rs::GemmP g{static_cast<const __half *>(a), static_cast<const __half *>(w), static_cast<__half *>(c),
                      static_cast<const __half *>(res), ws, counters, stats_in, colsum, stats_out, zero,
                      zero_len, m, n, k, eps, rope, bias};
    if (!rs::launch_gemm_epi(epi, g, sms, static_cast<cudaStream_t>(stream))) return -1;
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int jc_restated_attention(const void *qkv, void *o, uint32_t n, uint32_t window, uint32_t d, void *stream) {
    if (n < 1 || d % 64 || !qkv || !o) return -1;
    rs::attention_kernel<<<dim3((n + 63) / 64, d / 64), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half *>(qkv), static_cast<__half *>(o), n, window, d);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
