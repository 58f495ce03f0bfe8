// Kernel parameter blocks shared by the device code (.cuh) and the host runtime (.cpp): plain
// structs of device pointers and sizes.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace jc {

// Everything a GEMM reads or writes. The tensor maps are pointers: to the kernel's own parameters
// for a single launch, to a device array of maps for the persistent kernel.
struct GemmParams {
    const CUtensorMap *map_a;
    const CUtensorMap *map_w;
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

struct AttnParams {
    const __half *qkv;
    __half *o;
    float *ws;
    uint32_t *counters;
    uint32_t n, heads, window;
};

// Phase kinds of the persistent kernel.
enum : uint32_t {
    PH_GEMM = 0,
    PH_ATTN = 1,
    PH_EMBED = 2,     // out = LayerNorm(x[rows]) * gamma            (x: the embedding table)
    PH_NORM_ADD = 3,  // out = LayerNorm(x) * gamma + add, statistics
    PH_GATHER = 4,    // out = x[rows], stats = stats_in[rows]
    PH_SCORE = 5,     // logits = x[rows] . w + b
    PH_COPY = 6,      // out = x (n rows of d)
};

// A row-wise phase's operands.
struct RowParams {
    const __half *x;
    const uint32_t *rows;
    const float *gamma, *add, *stats_in;
    __half *out;
    float *stats, *logits;
    const __half *w;
    uint32_t n, d;
    float eps, b;
};

struct PhaseDesc {
    uint32_t kind, epi;
    GemmParams g;
    AttnParams a;
    RowParams r;
};

struct PersistParams {
    const PhaseDesc *phases;
    uint32_t n_phases;
    uint32_t *bar;        // [0] arrivals, [1] generation, [2] abort flag
    uint32_t expected;    // CTAs each grid barrier waits for (gridDim.x)
    uint64_t timeout_ns;
};

}  // namespace jc
