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
    const CUtensorMap *map_c;  // output tile through TMA stores (nullptr: direct stores)
    __half *c;
    const __half *res;
    float *ws;
    uint32_t *counters;
    const float *stats_in;
    const float *colsum;
    float *stats_out;
    float *zero;
    const float *rope;      // float4 [16][rope_stride]: (cos, sin) of pairs 2g, 2g + 1 of row r
    const float *bias;
    uint32_t rope_stride;   // rows of the RoPE table (>= m)
    uint32_t zero_len, m, n, k;
    float eps;
    uint32_t store_tma;     // single-GEMM kernel: the launch carries map_c
    // Packed requests (RoPE positions restart at each request): row r is position r - seg[r].x;
    // nullptr: position r.
    const uint2 *seg;
    // The error word device-side timeouts are recorded in (an engine's own); nullptr: the
    // module's word (jc_device_error).
    unsigned int *err;
    // A profiling run's phase stamps: prof_cap 8-word records, one per CTA (nullptr: none; the
    // single-GEMM kernel only).
    uint64_t *prof;
    uint32_t prof_cap;
};

struct AttnParams {
    const __half *qkv;
    __half *o;
    float *ws;
    uint32_t *counters;
    uint32_t n, heads, window;
    // Packed requests: row r belongs to the request occupying rows [seg[r].x, seg[r].y) and sees
    // only its keys; nullptr: one request of n rows.
    const uint2 *seg;
    unsigned int *err;  // error word (nullptr: the module's)
    uint64_t *prof;     // phase stamps of a profiling run (nullptr: none; standalone launches)
    uint32_t prof_cap;
    // Packed requests, tcgen05 kernel: CTA x takes query rows [tiles[x].x, tiles[x].y), at most
    // 128 rows of one request (empty entries: no work), attn_tile_cap(n) entries; nullptr: CTA x
    // takes rows [128 x, 128 x + 128).
    const uint2 *tiles;
};

// Entries of a packed forward's attention tile list: room for request-aligned tiles of up to 128
// rows when the requests average 128 rows or more (otherwise the list holds the plain 128-row
// tiles and the requests' keys still bound every query).
__host__ __device__ constexpr uint32_t attn_tile_cap(uint32_t n) { return 2 * ((n + 127) / 128); }

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
    uint32_t limit;  // marker gather: rows a marker may name (the head's rows)
};

// How a phase's items wait for an earlier phase: DEP_ROWS, the earlier phase's row block(s) that
// hold the item's own rows; DEP_WINDOW, those within `window` rows of them; DEP_ALL, every row
// block of the earlier phase.
enum : uint32_t { DEP_NONE = 0, DEP_ROWS = 1, DEP_WINDOW = 2, DEP_ALL = 3 };

struct PhaseDep {
    uint32_t kind;    // DEP_*
    uint32_t phase;   // index (within the launch) of the phase waited for
    uint32_t window;  // DEP_WINDOW: rows either side
};

// Rows are grouped in blocks of FLOW_BLOCK (the GEMM tile height): every finished item adds one to
// its block's completion counter, and a waiting item compares that counter with the number of
// items the block holds.
constexpr uint32_t FLOW_BLOCK = 128;
constexpr uint32_t FLOW_CHUNK = 32;  // query rows per attention item
constexpr uint32_t FLOW_ROWS = 8;    // rows per item of the row-wise phases (one per warp)

struct PhaseDesc {
    uint32_t kind, epi;
    uint32_t bn;  // GEMM phases: the persistent kernel's tile width (64, or 32), set by plan_flow
    GemmParams g;
    AttnParams a;
    RowParams r;
    // dataflow schedule (filled by the host)
    uint32_t rows;        // rows of this phase's output (the row space its counters cover)
    uint32_t items;       // work items: GEMM tiles (row-block major), attention (query chunk,
                          // head) pairs, or FLOW_ROWS-row chunks
    uint32_t first_item;  // global index of its first item within the launch
    uint32_t extra;       // added to every expected count of this phase (0; the timeout probe
                          // uses it to make a wait that cannot end)
    PhaseDep dep[2];
};

// The persistent kernel's launch: `ctr` holds n_phases x blocks completion counters followed by
// the work counter, the exit counter and the abort flag; all are zero between launches (the last
// CTA to leave clears them).
struct FlowParams {
    const PhaseDesc *phases;
    uint32_t n_phases, total_items, blocks;
    uint32_t *ctr;
    uint64_t timeout_ns;
    unsigned int *err;  // error word (nullptr: the module's)
    // A profiling run's phase stamps: record i (8 words) for the launch's item i < prof_cap
    // (nullptr: none).
    uint64_t *prof;
    uint32_t prof_cap;
};

}  // namespace jc
