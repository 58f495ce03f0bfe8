// The persistent kernel: one cooperative launch runs a list of phases (fused-epilogue GEMMs,
// attention, and the row-wise edges: embedding, head input, marker gather, score), every CTA
// striding over each phase's tasks, with a grid barrier between consecutive phases.
//
// It replaces the reference's persistent `layer` kernel (kernels/src/main.rs:579-826, host
// src/forward.rs:226-359): there, five phases of one encoder layer with the same tile code as the
// per-step kernels. Here the phase list is data (a device array of descriptors), so the same
// kernel runs one encoder layer per launch (the reference's layer-fused mode) or the whole model,
// embed to logits, in a single launch. B200 specifics:
//   - one CTA of 256 threads per SM holding the GEMM's TMEM accumulators and a 4-stage TMA ring
//     (8 k-blocks deep) for the whole launch (barriers initialised and TMEM allocated once);
//   - before each grid barrier the producer thread already requests the weight half of its first
//     stages of the next GEMM phase (weights never depend on the barrier), so the phase starts
//     with its weights on chip and only the activations left to fetch;
//   - the grid barrier is a counter plus a generation word (no reset between launches, so a CUDA
//     graph can replay it); every wait gives up after `timeout_ns`, records JC_DEV_TIMEOUT_GRID and
//     raises an abort flag that makes every other CTA leave at its next barrier.
#pragma once
#include "attention.cuh"
#include "edges.cuh"
#include "gemm_tile.cuh"
#include "params.h"

namespace jc {

constexpr int PERSIST_BN = 64;
constexpr int PERSIST_STAGES = 4;
using PersistGemm = GemmShape<PERSIST_BN, PERSIST_STAGES>;
using PersistAttn = AttnShape<2, 4>;
constexpr int PERSIST_THREADS = 256;
constexpr int PERSIST_SMEM = PersistGemm::SMEM_BYTES;
static_assert(PersistAttn::SMEM <= PersistGemm::STAGES * PersistGemm::STAGE_BYTES,
              "attention tasks reuse the GEMM stages' shared memory");
static_assert(PersistAttn::THREADS == PERSIST_THREADS && GEMM_THREADS == PERSIST_THREADS,
              "one CTA shape for every phase");

// Grid-wide barrier. Returns false if it (or another CTA's) timed out: the caller leaves.
__device__ __forceinline__ bool grid_barrier(uint32_t *bar, uint32_t expected, uint64_t timeout_ns) {
    __shared__ uint32_t ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile uint32_t *abort_flag = bar + 2;
        uint32_t gen;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
        __threadfence();
        const uint32_t old = atomicAdd(bar, 1u);
        bool ok = true;
        if (old == expected - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar + 1) : "memory");
        } else {
            const uint64_t t0 = globaltimer();
            while (true) {
                uint32_t now;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(now) : "l"(bar + 1) : "memory");
                if (now != gen) break;
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                if (globaltimer() - t0 > timeout_ns) {
                    dev_fail(JC_DEV_TIMEOUT_GRID);
                    *abort_flag = 1u;
                    __threadfence();
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
        ok_s = ok ? 1u : 0u;
    }
    __syncthreads();
    return ok_s != 0;
}

__device__ __forceinline__ uint32_t gemm_tiles(const GemmParams &g) {
    return (g.m + GEMM_BM - 1) / GEMM_BM * (g.n / PERSIST_BN);
}

template <uint32_t EPI>
__device__ __forceinline__ void persist_gemm(const GemmParams &g, const GemmSmemView<PERSIST_BN, PERSIST_STAGES> &sv,
                                             uint32_t tmem, GemmRun &run, uint32_t prefetched) {
    const uint32_t tiles_n = g.n / PERSIST_BN, tiles = gemm_tiles(g);
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x)
        gemm_tile<PERSIST_BN, PERSIST_STAGES, EPI>(g, sv, tmem, run, t % tiles_n, t / tiles_n, 0, 1,
                                                   t, t == blockIdx.x ? prefetched : 0, false);
}

__device__ __forceinline__ void persist_gemm_dispatch(uint32_t epi, const GemmParams &g,
                                                      const GemmSmemView<PERSIST_BN, PERSIST_STAGES> &sv,
                                                      uint32_t tmem, GemmRun &run, uint32_t pf) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    switch (epi) {
        case JC_EPI_ROPE: persist_gemm<JC_EPI_ROPE>(g, sv, tmem, run, pf); break;
        case JC_EPI_LN | JC_EPI_ROPE: persist_gemm<JC_EPI_LN | JC_EPI_ROPE>(g, sv, tmem, run, pf); break;
        case JC_EPI_LN | JC_EPI_GEGLU: persist_gemm<JC_EPI_LN | JC_EPI_GEGLU>(g, sv, tmem, run, pf); break;
        case RS: persist_gemm<RS>(g, sv, tmem, run, pf); break;
        case JC_EPI_BIAS | RS: persist_gemm<JC_EPI_BIAS | RS>(g, sv, tmem, run, pf); break;
        case LB: persist_gemm<LB>(g, sv, tmem, run, pf); break;
        case LB | JC_EPI_RELU: persist_gemm<LB | JC_EPI_RELU>(g, sv, tmem, run, pf); break;
        case LB | JC_EPI_GELU: persist_gemm<LB | JC_EPI_GELU>(g, sv, tmem, run, pf); break;
        default: dev_fail(JC_DEV_BAD_INDEX); break;
    }
}

// ---- row-wise phases: one warp per row, striding over every warp of the grid ----

// LayerNorm of a row of d f16 values (d a multiple of 128, at most 1024), then out = y * gamma +
// add (add optional), f16 out, and the stored values' sum / sum of squares into stats (optional).
__device__ __forceinline__ void ln_row(const __half *src, uint32_t d, const float *gamma,
                                       const float *add, float eps, __half *dst, float *stats,
                                       uint32_t lane) {
    float v[32];
    const uint32_t per = d / 128;
    const uint2 *s2 = reinterpret_cast<const uint2 *>(src);
    float sum = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 8; j++)
        if (j < per) {
            const uint2 q = s2[j * 32 + lane];
            const float2 a = unpack_half2(q.x), b = unpack_half2(q.y);
            v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = b.x; v[4 * j + 3] = b.y;
            sum += (a.x + a.y) + (b.x + b.y);
        }
    const float mean = warp_sum(sum) / d;
    float var = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 8; j++)
        if (j < per)
#pragma unroll
            for (int e = 0; e < 4; e++) var += (v[4 * j + e] - mean) * (v[4 * j + e] - mean);
    const float rstd = rsqrtf(warp_sum(var) / d + eps);
    uint2 *d2 = reinterpret_cast<uint2 *>(dst);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    const float4 *a4 = reinterpret_cast<const float4 *>(add);
    float s = 0.f, q2 = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 8; j++)
        if (j < per) {
            const float4 gm = __ldg(g4 + j * 32 + lane);
            const float4 ad = add ? __ldg(a4 + j * 32 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
            uint2 o;
            o.x = pack_half2((v[4 * j] - mean) * rstd * gm.x + ad.x,
                             (v[4 * j + 1] - mean) * rstd * gm.y + ad.y);
            o.y = pack_half2((v[4 * j + 2] - mean) * rstd * gm.z + ad.z,
                             (v[4 * j + 3] - mean) * rstd * gm.w + ad.w);
            d2[j * 32 + lane] = o;
            const float2 a = unpack_half2(o.x), b = unpack_half2(o.y);
            s += (a.x + a.y) + (b.x + b.y);
            q2 += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
        }
    if (stats) {
        s = warp_sum(s);
        q2 = warp_sum(q2);
        if (lane == 0) {
            stats[0] = s;
            stats[1] = q2;
        }
    }
}

__device__ __forceinline__ void persist_rows(uint32_t kind, const RowParams &r) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < r.n; i += warps) {
        if (kind == PH_EMBED) {
            ln_row(r.x + (size_t)r.rows[i] * r.d, r.d, r.gamma, nullptr, r.eps,
                   r.out + (size_t)i * r.d, r.stats ? r.stats + 2 * i : nullptr, lane);
        } else if (kind == PH_NORM_ADD) {
            ln_row(r.x + (size_t)i * r.d, r.d, r.gamma, r.add, r.eps, r.out + (size_t)i * r.d,
                   r.stats + 2 * i, lane);
        } else if (kind == PH_GATHER) {
            const uint32_t src = r.rows[i];
            const uint4 *s4 = reinterpret_cast<const uint4 *>(r.x + (size_t)src * r.d);
            uint4 *d4 = reinterpret_cast<uint4 *>(r.out + (size_t)i * r.d);
            for (uint32_t j = lane; j < r.d / 8; j += 32) d4[j] = s4[j];
            if (lane == 0) {
                r.stats[2 * i] = r.stats_in[2 * src];
                r.stats[2 * i + 1] = r.stats_in[2 * src + 1];
            }
        } else if (kind == PH_COPY) {
            const uint4 *s4 = reinterpret_cast<const uint4 *>(r.x + (size_t)i * r.d);
            uint4 *d4 = reinterpret_cast<uint4 *>(r.out + (size_t)i * r.d);
            for (uint32_t j = lane; j < r.d / 8; j += 32) d4[j] = s4[j];
        } else {  // PH_SCORE
            const uint32_t *row = reinterpret_cast<const uint32_t *>(r.x + (size_t)r.rows[i] * r.d);
            const uint32_t *wr = reinterpret_cast<const uint32_t *>(r.w);
            float acc = 0.f;
            for (uint32_t j = lane; j < r.d / 2; j += 32) {
                const float2 a = unpack_half2(row[j]), c = unpack_half2(__ldg(wr + j));
                acc = fmaf(a.x, c.x, acc);
                acc = fmaf(a.y, c.y, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) r.logits[i] = acc + r.b;
        }
    }
}

__global__ void __launch_bounds__(PERSIST_THREADS, 1) persist_kernel(const PersistParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const GemmSmemView<PERSIST_BN, PERSIST_STAGES> sv(base);
    const uint32_t tmem = gemm_setup<PERSIST_BN, PERSIST_STAGES>(sv);
    GemmRun run;
    pdl_wait();
    pdl_launch_dependents();
    uint32_t prefetched = 0;
    for (uint32_t ph = 0; ph < P.n_phases; ph++) {
        const PhaseDesc &d = P.phases[ph];
        const uint32_t kind = d.kind;
        if (kind == PH_GEMM) {
            persist_gemm_dispatch(d.epi, d.g, sv, tmem, run, prefetched);
            gemm_zero(d.g, blockIdx.x, gridDim.x);
        } else if (kind == PH_ATTN) {
            const uint32_t qtiles = (d.a.n + PersistAttn::QT - 1) / PersistAttn::QT;
            const uint32_t tasks = qtiles * d.a.heads;
            for (uint32_t t = blockIdx.x; t < tasks; t += gridDim.x)
                attention_task<2, 4>(d.a, base, t / d.a.heads, t % d.a.heads, 0, 1, false);
        } else {
            persist_rows(kind, d.r);
        }
        prefetched = 0;
        if (ph + 1 == P.n_phases) break;
        // Hand the shared memory from the generic proxy (attention, row phases) to TMA.
        fence_proxy_async();
        __syncthreads();
        const PhaseDesc &nx = P.phases[ph + 1];
        if (nx.kind == PH_GEMM && blockIdx.x < gemm_tiles(nx.g)) {
            const uint32_t nst = gemm_stages(nx.g.k / GEMM_BK);
            prefetched = nst < (uint32_t)PERSIST_STAGES ? nst : (uint32_t)PERSIST_STAGES;
            if (threadIdx.x == 0) {
                tma_prefetch_desc(nx.g.map_a);
                tma_prefetch_desc(nx.g.map_w);
                const uint32_t tiles_n = nx.g.n / PERSIST_BN;
                gemm_issue_w<PERSIST_BN, PERSIST_STAGES>(nx.g, sv, run.it,
                                                         (blockIdx.x % tiles_n) * PERSIST_BN, 0, 0,
                                                         prefetched);
            }
        }
        if (!grid_barrier(P.bar, P.expected, P.timeout_ns)) {
            // Leaving early: complete the stages whose weights are already in flight (their A
            // halves too, so the stage barriers can finish) and wait for them, within limits.
            if (threadIdx.x == 0 && prefetched) {
                const uint32_t tiles_n = nx.g.n / PERSIST_BN;
                const uint32_t m0 = (blockIdx.x / tiles_n) * GEMM_BM;
                for (uint32_t i = 0; i < prefetched; i++)
                    gemm_issue_a<PERSIST_BN, PERSIST_STAGES>(nx.g, sv, run.it, m0, 0, i);
                for (uint32_t i = 0; i < prefetched; i++) {
                    const uint32_t g = run.it + i;
                    mbar_wait(&sv.full[g % PERSIST_STAGES], (g / PERSIST_STAGES) & 1,
                              JC_DEV_TIMEOUT_FULL);
                }
            }
            break;
        }
        // Activations written by other CTAs before the barrier are read by TMA after it.
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    gemm_teardown<PERSIST_BN, PERSIST_STAGES>(tmem);
}

}  // namespace jc
