// Device helpers shared by the sm_100a kernels: mbarriers with bounded waits, TMA tiled loads,
// tcgen05 (TMEM alloc / MMA / commit / ld), programmatic dependent launch, f16 packing.
//
// Every wait here is bounded: a wait that runs past its limit records an error code in the
// module's error word (read by the host after each call) and gives up, so a bug can never hang a
// shared GPU.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "jc_internal.h"

namespace jc {

// The module-wide error word: 0, or the first JC_DEV_* code a kernel recorded. It serves the
// per-kernel entry points (jc_gemm, jc_attention, ...), which have no engine; an engine passes
// its own word in every launch's parameters, so two engines on one GPU (or an engine beside bare
// jc_* calls) never see or clear each other's errors. (All kernels live in one translation unit,
// kernels.cu, so this is the only definition.)
__device__ unsigned int g_dev_error = 0;

// The word the running CTA records errors into. Every kernel that can record an error binds it
// first thing (dev_err_bind, by every thread: each writes the same value, so no barrier is
// needed before its own later reads).
__shared__ unsigned int *s_dev_err;

__device__ __forceinline__ void dev_err_bind(unsigned int *word) {
    s_dev_err = word ? word : &g_dev_error;
}

__device__ __forceinline__ void dev_fail(unsigned int code) { atomicCAS(s_dev_err, 0u, code); }

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Optional per-CTA phase stamps of a profiling run (off unless a launch passes a record array):
// 8 words a CTA, [0] entry, [1] inputs ready (the previous kernel done), [2] first operand stage
// in shared memory, [3] results complete (accumulator / key loop), [4] outputs written, [5] exit
// (%globaltimer ns; 0 where a stage does not apply), [6] the SM, [7] the CTA's linear index.
__device__ __forceinline__ uint64_t *prof_record(uint64_t *prof, uint32_t cap) {
    if (!prof) return nullptr;
    if (cap == 0) return prof;  // the persistent kernel's item: prof is the item's own record
    const uint32_t cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    return cta < cap ? prof + 8 * (size_t)cta : nullptr;
}

__device__ __forceinline__ void prof_stamp(uint64_t *rec, int slot) {
    if (rec) rec[slot] = globaltimer();
}

__device__ __forceinline__ void prof_open(uint64_t *rec) {
    if (!rec) return;
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    rec[0] = globaltimer();
    rec[1] = rec[2] = rec[3] = rec[4] = rec[5] = 0;
    rec[6] = sm;
    rec[7] = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread (up to `hint_ns`) until the phase completes,
// instead of spinning on the issue slots the working warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity,
                                                    uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with this parity to complete; gives up after ~JC_WAIT_NS and
// records `code`. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        for (int i = 0; i < 16; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > JC_WAIT_NS) {
            dev_fail(code);
            return false;
        }
    }
}

// The same for threads with nothing else to do meanwhile: suspended between polls.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity,
                                                unsigned int code) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait_sleep(bar, parity, 200000u)) {
        if (globaltimer() - t0 > JC_WAIT_NS) {
            dev_fail(code);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of the box at (x = inner coordinate, y = row) into smem, completing on `bar`.
// x * sizeof(element) must be a multiple of 16 bytes (callers pass multiples of 64 f16).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 3-D tiled load at (x, y, z) (GEMM operands: x the column inside a 64-wide k-block, always 0;
// y the row; z the k-block), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 2-D tiled store of the box at smem `src` to (x = column, y = row) of the tensor; elements
// outside the tensor are not written. x * sizeof(element) must be a multiple of 16 bytes and
// neither coordinate negative (callers pass tile origins). Completes as a bulk async group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int32_t x,
                                             int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the bulk stores committed so far have read their shared memory.
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// programmatic dependent launch (no-ops when the launch has no PDL attribute)

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05

// Allocates `ncols` TMEM columns (a power of two >= 32); the whole warp calls it. The base address
// is written to `*slot` (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16 inputs, f32 accumulator).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 16 / 8 / 4 consecutive f32 columns of this thread's TMEM lane into v.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float *v);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float *v) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive f32 columns of this thread's TMEM lane (warp w reads lanes 32(w%4)..+31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major tile whose rows are 128 bytes (64 f16), swizzled
// with the 128-byte pattern in 1024-byte groups of 8 rows (what TMA's SWIZZLE_128B writes):
// start >> 4 in bits 0-13, leading byte offset (unused for this layout, 16) in 16-29, stride
// byte offset (1024: the next 8-row group) in 32-45, descriptor version 1 in 46-47, swizzle mode
// 2 (128B) in 61-63. `saddr` must be 1024-byte aligned for the base offset (49-51) to be 0.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(16 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with f16 A and B (both K-major), f32 accumulator, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4)                        // accumulator format: f32
           | (0u << 7) | (0u << 10)         // A, B: f16
           | ((uint32_t)(N >> 3) << 17)     // N / 8
           | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------------------------
// misc

// The keys query row q may see, [lo, hi] inclusive: its request's rows (seg[q] for packed
// requests, else [0, n)) and, with a window, those within `window` of q.
__device__ __forceinline__ void key_span(const uint2 *seg, uint32_t n, uint32_t window, uint32_t q,
                                         int &lo, int &hi) {
    int s0 = 0, s1 = (int)n;
    if (seg) {
        const uint2 sg = seg[q < n ? q : n - 1];
        s0 = (int)sg.x;
        s1 = (int)sg.y;
    }
    lo = s0;
    hi = s1 - 1;
    if (window) {
        lo = max(lo, (int)q - (int)window);
        hi = min(hi, (int)q + (int)window);
    }
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

// 2^x on the special-function unit (PTX ex2.approx.ftz; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU(x) = x * Phi(x) with Phi from the Abramowitz & Stegun 7.1.26 erf approximation (the
// formula julia-rs and the reference kernels use; kernels/src/gemm.rs:139-150). The reciprocal is
// the hardware approximation (a couple of ulp; the result's error stays near 1e-7 relative).
__device__ __forceinline__ float gelu_as(float x) {
    float t = __fdividef(1.0f, 1.0f + 0.2316419f * fabsf(x));
    float p = 0.5f * 1.061405429f;
    p = p * t + 0.5f * -1.453152027f;
    p = p * t + 0.5f * 1.421413741f;
    p = p * t + 0.5f * -0.284496736f;
    p = p * t + 0.5f * 0.254829592f;
    float q = p * t * __expf(-0.5f * x * x);
    return x * (x >= 0.0f ? 1.0f - q : q);
}

// p[0] += a, p[1] += b as one vector reduction (p 8-byte aligned), no return value.
__device__ __forceinline__ void red_add_f32x2(float *p, float a, float b) {
    asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b)
                 : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace jc
