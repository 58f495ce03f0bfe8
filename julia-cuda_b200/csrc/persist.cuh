// The persistent kernel: one cooperative launch runs a list of phases (fused-epilogue GEMMs,
// attention, and the row-wise edges: embedding, head input, marker gather, score) as a dataflow
// graph of work items, with no grid-wide barrier.
//
// It replaces the reference's persistent `layer` kernel (kernels/src/main.rs:579-826, host
// src/forward.rs:226-359), which runs five phases of one encoder layer separated by grid barriers.
// Here the phase list is data (a device array of descriptors), so the same kernel runs one encoder
// layer per launch (the reference's layer-fused mode) or the whole model, embed to logits, in a
// single launch. B200 specifics:
//   - one CTA of 256 threads per SM holds the GEMM's TMEM accumulators and a 4-stage TMA ring for
//     the whole launch (barriers initialised and TMEM allocated once);
//   - items (GEMM tiles, row-block major; (32-query chunk, head) attention tasks; 8-row chunks of
//     the row-wise phases, one row per warp) are handed out in phase order by one atomic counter,
//     a CTA taking its next item when it has finished the current one;
//   - an item waits only for the rows it reads: each finished item adds one to its 128-row block's
//     completion counter (a release reduction), and an item's TMA thread polls the counters of the
//     blocks it depends on (acquire loads; same block, a window of blocks for sliding-window
//     attention, every block for global attention and the marker gather). A GEMM tile requests its
//     weights before it waits, so they stream in while the producing phase finishes;
//   - items are taken in order and every CTA is resident, so the lowest unfinished item always has
//     its inputs: no deadlock. Every wait gives up after `timeout_ns`, records JC_DEV_TIMEOUT_GRID
//     and raises an abort flag that makes every other CTA leave;
//   - the last CTA to leave clears every counter, so a CUDA graph can replay the launch.
#pragma once
#include "attention.cuh"
#include "edges.cuh"
#include "gemm_tile.cuh"
#include "params.h"

namespace jc {

// GEMM phases run 64-column tiles, or 32-column ones where the plan (plan_flow) finds them
// cheaper: both share the stage memory; each has its own barriers and pipeline position.
constexpr int PERSIST_BN = 64;
constexpr int PERSIST_STAGES = 4;
constexpr int PERSIST_BN_NARROW = 32;
constexpr int PERSIST_STAGES_NARROW = 4;
using PersistGemm = GemmShape<PERSIST_BN, PERSIST_STAGES>;
using PersistGemmNarrow = GemmShape<PERSIST_BN_NARROW, PERSIST_STAGES_NARROW>;
constexpr uint32_t PERSIST_TAIL = PERSIST_STAGES * PersistGemm::STAGE_BYTES;
constexpr uint32_t PERSIST_NARROW_BAR_OFF = 128;  // the narrow view's barriers in the shared tail
static_assert(PERSIST_STAGES_NARROW * PersistGemmNarrow::STAGE_BYTES <= (int)PERSIST_TAIL,
              "the narrow tiles' stages fit the wide ones' stage memory");
static_assert(PERSIST_NARROW_BAR_OFF + 8 * (2 * PERSIST_STAGES_NARROW + 3) <= 256 &&
                  8 * (2 * PERSIST_STAGES + 3) <= (int)PERSIST_NARROW_BAR_OFF,
              "both views' barriers fit the tail's barrier block");
static_assert(PersistGemm::NI * PERSIST_BN >= PersistGemmNarrow::NI * PERSIST_BN_NARROW,
              "the narrow tiles' accumulators fit the TMEM allocated for the wide ones");
using PersistAttn = AttnShape<2, 4>;
constexpr int PERSIST_THREADS = 256;
constexpr int PERSIST_SMEM = PersistGemm::SMEM_BYTES;
static_assert(PersistAttn::SMEM <= PersistGemm::STAGES * PersistGemm::STAGE_BYTES,
              "attention tasks reuse the GEMM stages' shared memory");
static_assert(PersistAttn::THREADS == PERSIST_THREADS && GEMM_THREADS == PERSIST_THREADS,
              "one CTA shape for every phase");
static_assert(PersistAttn::QT == FLOW_CHUNK && FLOW_BLOCK == GEMM_BM && FLOW_BLOCK % FLOW_CHUNK == 0 &&
                  FLOW_ROWS == PERSIST_THREADS / 32 && FLOW_BLOCK % FLOW_ROWS == 0,
              "attention chunks, row chunks and GEMM row blocks tile the flow blocks");
static_assert(sizeof(PhaseDesc) % 4 == 0, "descriptors are copied to shared memory as words");

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Items of phase d that report to row block b (what a waiting item compares the counter with).
__device__ __forceinline__ uint32_t block_items(const PhaseDesc &d, uint32_t b) {
    const uint32_t r0 = b * FLOW_BLOCK;
    if (r0 >= d.rows) return d.extra;
    const uint32_t r1 = min(r0 + FLOW_BLOCK, d.rows);
    uint32_t c;
    if (d.kind == PH_GEMM)
        c = d.g.n / d.bn;
    else if (d.kind == PH_ATTN)
        c = (r1 - r0 + FLOW_CHUNK - 1) / FLOW_CHUNK * d.a.heads;
    else
        c = (r1 - r0 + FLOW_ROWS - 1) / FLOW_ROWS;
    return c + d.extra;
}

// TMA thread of an item covering rows [r0, r1): waits until the phase `dep` names has finished
// every item those rows read. false if the wait timed out (or another CTA's did).
__device__ __noinline__ bool wait_dep(const FlowParams &F, const PhaseDep &dep, uint32_t r0, uint32_t r1) {
    if (dep.kind == DEP_NONE) return true;
    const PhaseDesc &src = F.phases[dep.phase];
    const uint32_t nb = (src.rows + FLOW_BLOCK - 1) / FLOW_BLOCK;
    uint32_t b0 = 0, b1 = nb;
    if (dep.kind != DEP_ALL) {
        const uint32_t w = dep.kind == DEP_WINDOW ? dep.window : 0;
        b0 = (r0 > w ? r0 - w : 0) / FLOW_BLOCK;
        b1 = min((r1 + w + FLOW_BLOCK - 1) / FLOW_BLOCK, nb);
    }
    const uint32_t *ctr = F.ctr + dep.phase * F.blocks;
    volatile uint32_t *abort_flag = F.ctr + F.n_phases * F.blocks + 2;
    const uint64_t t0 = globaltimer();
    for (uint32_t b = b0; b < b1; b++) {
        const uint32_t want = block_items(src, b);
        while (ld_acquire_u32(ctr + b) < want) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > F.timeout_ns) {
                dev_fail(JC_DEV_TIMEOUT_GRID);
                *abort_flag = 1u;
                __threadfence();
                return false;
            }
        }
    }
    return true;
}

// The TMA thread waits for both dependencies of an item; generic-proxy writes of other CTAs are
// then ordered before this CTA's TMA reads.
__device__ __forceinline__ bool wait_item(const FlowParams &F, const PhaseDesc &d, uint32_t r0, uint32_t r1) {
    const bool ok = wait_dep(F, d.dep[0], r0, r1) && wait_dep(F, d.dep[1], r0, r1);
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return ok;
}

// A profiling run's record of the launch's item `item` (nullptr: none).
__device__ __forceinline__ uint64_t *item_record(const FlowParams *F, uint32_t item) {
    return F->prof && item < F->prof_cap ? F->prof + 8 * (size_t)item : nullptr;
}

// gemm_tile's gate in the persistent kernel: the TMA thread waits for the tile's row block; the
// other threads wait for it at a CTA barrier.
struct FlowGate {
    const FlowParams *F;
    const PhaseDesc *d;
    uint32_t r0, r1;
    uint32_t *ok_s;
    __device__ void producer() const { *ok_s = wait_item(*F, *d, r0, r1) ? 1u : 0u; }
    __device__ void all() const { __syncthreads(); }
};

// One GEMM tile of the current phase. Everything the tile code reads repeatedly is a local value
// here (parameters copied out of shared memory, the shared-memory view rebuilt from its base, the
// pipeline position passed in and returned), so it stays in registers across the tile's fences.
template <uint32_t EPI, int BN = PERSIST_BN>
__device__ __noinline__ uint2 flow_gemm_tile(const FlowParams *F, const PhaseDesc *d, uint8_t *base,
                                             uint32_t tmem, uint2 pos, uint32_t tm, uint32_t tn,
                                             uint32_t *ok_s) {
    constexpr int STAGES = BN == PERSIST_BN ? PERSIST_STAGES : PERSIST_STAGES_NARROW;
    GemmParams g = d->g;
    g.prof = item_record(F, d->first_item + tm * (g.n / BN) + tn);
    g.prof_cap = 0;
    const GemmSmemView<BN, STAGES> sv(base, PERSIST_TAIL, BN == PERSIST_BN ? 0 : PERSIST_NARROW_BAR_OFF);
    GemmRun run;
    run.it = pos.x;
    run.tiles = pos.y;
    const FlowGate gate{F, d, tm * GEMM_BM, min((tm + 1) * GEMM_BM, d->rows), ok_s};
    gemm_tile<BN, STAGES, EPI>(g, sv, tmem, run, tn, tm, 0, 1, 0, 0, gate);
    return make_uint2(run.it, run.tiles);
}

// A narrow (32-column) tile of the epilogues that allow one (not RoPE or GeGLU, whose pairs span
// 64 columns). pos: the narrow view's pipeline position.
__device__ __forceinline__ uint2 flow_gemm_narrow(const FlowParams *F, const PhaseDesc *d, uint8_t *base,
                                                  uint32_t tmem, uint2 pos, uint32_t tm, uint32_t tn,
                                                  uint32_t *ok_s) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    constexpr int NB = PERSIST_BN_NARROW;
    switch (d->epi) {
        case RS: return flow_gemm_tile<RS, NB>(F, d, base, tmem, pos, tm, tn, ok_s);
        case JC_EPI_BIAS | RS: return flow_gemm_tile<JC_EPI_BIAS | RS, NB>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB: return flow_gemm_tile<LB, NB>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB | JC_EPI_RELU: return flow_gemm_tile<LB | JC_EPI_RELU, NB>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB | JC_EPI_GELU: return flow_gemm_tile<LB | JC_EPI_GELU, NB>(F, d, base, tmem, pos, tm, tn, ok_s);
        default:
            if (threadIdx.x == 0) {
                dev_fail(JC_DEV_BAD_INDEX);
                *ok_s = 0u;
            }
            __syncthreads();
            return pos;
    }
}

__device__ __forceinline__ uint2 flow_gemm(const FlowParams *F, const PhaseDesc *d, uint8_t *base,
                                           uint32_t tmem, uint2 pos, uint32_t tm, uint32_t tn,
                                           uint32_t *ok_s) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    switch (d->epi) {
        case JC_EPI_ROPE: return flow_gemm_tile<JC_EPI_ROPE>(F, d, base, tmem, pos, tm, tn, ok_s);
        case JC_EPI_LN | JC_EPI_ROPE: return flow_gemm_tile<JC_EPI_LN | JC_EPI_ROPE>(F, d, base, tmem, pos, tm, tn, ok_s);
        case JC_EPI_LN | JC_EPI_GEGLU: return flow_gemm_tile<JC_EPI_LN | JC_EPI_GEGLU>(F, d, base, tmem, pos, tm, tn, ok_s);
        case RS: return flow_gemm_tile<RS>(F, d, base, tmem, pos, tm, tn, ok_s);
        case JC_EPI_BIAS | RS: return flow_gemm_tile<JC_EPI_BIAS | RS>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB: return flow_gemm_tile<LB>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB | JC_EPI_RELU: return flow_gemm_tile<LB | JC_EPI_RELU>(F, d, base, tmem, pos, tm, tn, ok_s);
        case LB | JC_EPI_GELU: return flow_gemm_tile<LB | JC_EPI_GELU>(F, d, base, tmem, pos, tm, tn, ok_s);
        default:
            // Unknown epilogue (the host never builds one): record it and leave the tile undone.
            if (threadIdx.x == 0) {
                dev_fail(JC_DEV_BAD_INDEX);
                *ok_s = 0u;
            }
            __syncthreads();
            return pos;
    }
}

// One attention task of the current phase, its parameters as local values.
__device__ __noinline__ void flow_attention(const PhaseDesc *d, uint8_t *base, uint32_t chunk,
                                            uint32_t head, uint64_t *rec) {
    AttnParams a = d->a;
    a.prof = rec;
    a.prof_cap = 0;
    attention_task<2, 4>(a, base, chunk, head, 0, 1, false);
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

// Row i of a row-wise phase, by one warp.
__device__ __noinline__ void row_op(uint32_t kind, const RowParams &r, uint32_t i, uint32_t lane) {
    if (kind == PH_EMBED) {
        ln_row(r.x + (size_t)r.rows[i] * r.d, r.d, r.gamma, nullptr, r.eps,
               r.out + (size_t)i * r.d, r.stats ? r.stats + 2 * i : nullptr, lane);
    } else if (kind == PH_NORM_ADD) {
        ln_row(r.x + (size_t)i * r.d, r.d, r.gamma, r.add, r.eps, r.out + (size_t)i * r.d,
               r.stats + 2 * i, lane);
    } else if (kind == PH_GATHER) {
        const uint32_t src = r.rows[i];
        if (src >= r.limit) {
            if (lane == 0) dev_fail(JC_DEV_BAD_INDEX);
            return;
        }
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

__global__ void __launch_bounds__(PERSIST_THREADS, 1) persist_kernel(const __grid_constant__ FlowParams F) {
    dev_err_bind(F.err);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    __shared__ uint32_t item_s[2], ok_s;
    // The current item's descriptor: read from shared memory, not global memory (the item's code
    // reads its parameters many times, across fences that would force global reloads).
    __shared__ __align__(16) PhaseDesc desc_s;
    gemm_init_barriers<PERSIST_BN_NARROW, PERSIST_STAGES_NARROW>(
        GemmSmemView<PERSIST_BN_NARROW, PERSIST_STAGES_NARROW>(base, PERSIST_TAIL, PERSIST_NARROW_BAR_OFF));
    const uint32_t tmem = gemm_setup<PERSIST_BN, PERSIST_STAGES>(GemmSmemView<PERSIST_BN, PERSIST_STAGES>(base));
    // The two GEMM pipelines' positions (GemmRun) across tiles: 64-column and 32-column tiles.
    uint2 pos = make_uint2(0, 0), pos_narrow = make_uint2(0, 0);
    pdl_wait();
    pdl_launch_dependents();
    uint32_t *work = F.ctr + F.n_phases * F.blocks;  // then the exit counter, the abort flag
    uint32_t next = 0;
    if (threadIdx.x == 0) next = atomicAdd(work, 1u);
    uint32_t ph = 0, desc_ph = 0;
    for (uint32_t iter = 0;; iter++) {
        if (threadIdx.x == 0) {
            item_s[iter & 1] = next;
            // Profiling runs: the item's record is opened before any thread of the CTA stamps it.
            if (uint64_t *rec = next < F.total_items ? item_record(&F, next) : nullptr) {
                uint32_t sm;
                asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
                rec[0] = globaltimer();
                rec[1] = rec[2] = rec[3] = rec[4] = rec[5] = 0;
                rec[6] = sm;
                rec[7] = blockIdx.x;
            }
        }
        __syncthreads();
        const uint32_t item = item_s[iter & 1];
        if (item >= F.total_items) break;
        while (item >= F.phases[ph].first_item + F.phases[ph].items) ph++;
        if (iter == 0 || ph != desc_ph) {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(F.phases + ph);
            uint32_t *dst = reinterpret_cast<uint32_t *>(&desc_s);
            for (uint32_t i = threadIdx.x; i < sizeof(PhaseDesc) / 4; i += PERSIST_THREADS) dst[i] = src[i];
            desc_ph = ph;
            if (threadIdx.x == 0 && F.phases[ph].kind == PH_GEMM) {
                tma_prefetch_desc(F.phases[ph].g.map_a);
                tma_prefetch_desc(F.phases[ph].g.map_w);
            }
            __syncthreads();
        }
        const PhaseDesc &d = desc_s;
        const uint32_t local = item - d.first_item;
        uint32_t block;
        if (d.kind == PH_GEMM) {
            const uint32_t tiles_n = d.g.n / d.bn;
            const uint32_t tm = local / tiles_n, tn = local % tiles_n;
            block = tm;
            if (d.bn == PERSIST_BN_NARROW)
                pos_narrow = flow_gemm_narrow(&F, &desc_s, base, tmem, pos_narrow, tm, tn, &ok_s);
            else
                pos = flow_gemm(&F, &desc_s, base, tmem, pos, tm, tn, &ok_s);
            // The first tile of a row block clears that block's rows of the statistics buffer a
            // later GEMM adds into (its readers are done: they precede this tile's inputs).
            if (tn == 0 && d.g.zero)
                for (uint32_t i = tm * 2 * GEMM_BM + threadIdx.x; i < min((tm + 1) * 2 * GEMM_BM, d.g.zero_len);
                     i += PERSIST_THREADS)
                    d.g.zero[i] = 0.0f;
        } else {
            const uint32_t rows = d.kind == PH_ATTN ? FLOW_CHUNK : FLOW_ROWS;
            const uint32_t chunk = d.kind == PH_ATTN ? local / d.a.heads : local;
            block = chunk * rows / FLOW_BLOCK;
            const uint32_t r0 = chunk * rows, r1 = min(r0 + rows, d.rows);
            uint64_t *rec = threadIdx.x == 0 ? item_record(&F, item) : nullptr;
            if (threadIdx.x == 0) {
                ok_s = wait_item(F, d, r0, r1) ? 1u : 0u;
                prof_stamp(rec, 1);
            }
            __syncthreads();
            if (ok_s) {
                if (d.kind == PH_ATTN) {
                    flow_attention(&desc_s, base, chunk, local % d.a.heads, rec);
                } else {
                    const uint32_t lane = threadIdx.x & 31;
                    for (uint32_t i = r0 + (threadIdx.x >> 5); i < r1; i += PERSIST_THREADS / 32)
                        row_op(d.kind, d.r, i, lane);
                }
                // Hand the shared memory from the generic proxy back to TMA.
                fence_proxy_async();
            }
        }
        __syncthreads();
        if (!ok_s) break;
        // Report the item, then take the next one (taken only now: an item held by a busy CTA
        // could not start on an idle one; taking it one ahead, as the current one starts,
        // measured 1353 against 1056 us for the whole model at 293 tokens).
        if (threadIdx.x == 0) {
            red_release_add(F.ctr + ph * F.blocks + block, 1u);
            prof_stamp(item_record(&F, item), 5);
            next = atomicAdd(work, 1u);
        }
    }
    gemm_teardown<PERSIST_BN, PERSIST_STAGES>(tmem);
    // The last CTA to leave clears every counter for the next launch.
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(work + 1, 1u);
        ok_s = old == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (ok_s) {
        __threadfence();
        for (uint32_t i = threadIdx.x; i < F.n_phases * F.blocks + 3; i += PERSIST_THREADS) F.ctr[i] = 0u;
    }
}

}  // namespace jc
