// Internal declarations shared by the kernels (.cu) and the host runtime (.cpp).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "../../include/julia_cuda.h"

// Longest a device-side wait may spin before it records an error and gives up (ns).
#define JC_WAIT_NS 2000000000ull

// Device error codes (the module error word holds the first one recorded).
#define JC_DEV_TIMEOUT_FULL 1u     // MMA issuer: a TMA stage never arrived
#define JC_DEV_TIMEOUT_EMPTY 2u    // TMA producer: a stage was never released by the MMAs
#define JC_DEV_TIMEOUT_MMA 3u      // epilogue: the accumulator was never committed
#define JC_DEV_TIMEOUT_GRID 4u     // persistent kernel: a grid barrier timed out
#define JC_DEV_TIMEOUT_SPLIT 5u    // split-K / split-KV: partials never became complete
#define JC_DEV_BAD_INDEX 6u        // an index a kernel checks was out of range

// GEMM epilogue flags: JC_EPI_* from the public header (the reference's bit values,
// kernels/src/main.rs:870-877).

namespace jc {

// Thread-local last error message of the C ABI.
void set_error(const std::string &msg);
const char *last_error();

// Records a CUDA error; returns false if `e` is an error.
bool cuda_ok(cudaError_t e, const char *what);

// ---------------------------------------------------------------------------------------------
// TMA descriptors

// A row-major [rows, cols] f16 GEMM operand (cols a multiple of 64) seen as 3-D: (column inside a
// 64-wide k-block, row, k-block), loaded in boxes of 64 x box_rows x GEMM_KPS with the 128-byte
// swizzle, so one box lands as GEMM_KPS consecutive [box_rows][128 B] k-block tiles. Returns false
// (and sets the error) on failure. A GEMM's A operand takes boxes of its tile height
// (GemmConfig::bm), its W operand boxes of its tile width (GemmConfig::bn).
bool make_tmap_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                   uint32_t box_rows);

// ---------------------------------------------------------------------------------------------
// GEMM: c = epilogue(a . w^T), a [m,k] f16, w [n,k] f16, tcgen05 with TMEM accumulators.

struct GemmArgs {
    uint32_t epi = 0;
    CUtensorMap map_a{}, map_w{};
    __half *c = nullptr;
    const __half *res = nullptr;
    float *ws = nullptr;
    uint32_t *counters = nullptr;
    const float *stats_in = nullptr;
    const float *colsum = nullptr;
    float *stats_out = nullptr;
    float *zero = nullptr;
    uint32_t zero_len = 0;
    uint32_t m = 0, n = 0, k = 0;
    float eps = 0.f;
    const float *rope = nullptr;
    const float *bias = nullptr;
    uint32_t rope_stride = 0;  // rows of the pair-group-major RoPE table; 0: m
    const uint2 *seg = nullptr;  // packed requests: row r's request rows (RoPE position r - seg[r].x)
    unsigned int *err = nullptr;  // error word for device-side timeouts (nullptr: the module's)
    uint64_t *prof = nullptr;     // profiling run: per-CTA phase stamps (8 words a CTA)
    uint32_t prof_cap = 0;        // records available at prof
};

struct GemmConfig {
    int bm = 128;     // output rows per CTA: 128, or 64 (32- and 64-column tiles, no split-K)
    int bn = 64;      // output columns per CTA: 32, 64, 128 or 256
    int splits = 1;   // split-K factor through a global workspace, 1..8
    int cluster = 1;  // split-K factor inside a thread-block cluster (1, 2 or 4; DSMEM reduction)
    bool deep = false;  // twice the pipeline stages (one CTA per SM)
    // More tiles than SMs, 128- or 256-column tiles, no split: one CTA per SM walks the tiles
    // with the epilogue of one under the main loop of the next (gemm_persist.cuh) on `grid` CTAs.
    bool persistent = false;
    uint32_t grid = 0;
    // CTA pairs (gemm_pair.cuh): 256 x bn tiles, a cluster of two CTAs each holding 128 rows
    // and half of the weight rows (its W tensor map's box is bn / 2 rows: gemm_w_rows).
    bool pair = false;
};

// Rows of the W tensor map's box for a configuration: the tile width, or half of it for pairs.
inline uint32_t gemm_w_rows(const GemmConfig &c) { return (uint32_t)(c.pair ? c.bn / 2 : c.bn); }
// CTA-pair policy (1 always where legal, 0 automatic, -1 never): sets it, returns the old one.
void swap_gemm_pair_policy(int *policy);

// Floats of split-K workspace and counters a launch of this shape needs.
size_t gemm_ws_floats(uint32_t m, uint32_t n, GemmConfig cfg);
size_t gemm_counters(uint32_t m, uint32_t n, GemmConfig cfg);

// Validates and launches; false (with the error set) if the arguments are inconsistent.
bool launch_gemm(const GemmArgs &g, GemmConfig cfg, cudaStream_t s, bool pdl);
// The argument checks alone (the tensor maps are not looked at).
bool check_gemm(const GemmArgs &g, GemmConfig cfg);

// The configuration for an m x n x k GEMM on `sms` SMs (the B200 refit of gemm::choose).
GemmConfig choose_gemm(uint32_t m, uint32_t n, uint32_t k, int sms);
// A caller's split-K request: > 0 that many splits through the workspace, < 0 a cluster of -splits
// CTAs reducing through distributed shared memory (no workspace), 0 keeps the automatic choice.
void request_splits(GemmConfig &c, int splits);
// Picks the tile height and pipeline depth for a configuration whose tile width / splits are
// already set.
void set_gemm_depth(GemmConfig &c, uint32_t m, uint32_t n, int sms);
// The tile height policy (0 automatic, 128, or 64 wherever legal): sets it, returns the old one.
void swap_gemm_tile_rows(int *rows);

// ---------------------------------------------------------------------------------------------
// attention: o = softmax(q k^T / 8) v per head, global or |q - k| <= window

struct AttnArgs {
    const __half *qkv = nullptr;  // [n, 3 * heads * 64]
    __half *o = nullptr;          // [n, heads * 64]
    uint32_t n = 0, heads = 0, window = 0;
    uint32_t kv_chunks = 1;       // split-KV: key ranges per (query tile, head)
    float *ws = nullptr;          // kv_chunks > 1: partials
    uint32_t *counters = nullptr; // kv_chunks > 1: one zeroed counter per (query tile, head)
    const uint2 *seg = nullptr;   // packed requests: row r sees only keys [seg[r].x, seg[r].y)
    unsigned int *err = nullptr;  // error word (nullptr: the module's)
    uint64_t *prof = nullptr;     // profiling run: per-CTA phase stamps (8 words a CTA)
    uint32_t prof_cap = 0;
    // packed requests: the tcgen05 kernel's request-aligned tiles (attn_tile_cap(n) entries)
    const uint2 *tiles = nullptr;
};
size_t attn_ws_floats(uint32_t n, uint32_t heads, uint32_t kv_chunks);
// CTAs a launch_attention of these arguments runs.
uint32_t attention_ctas(const AttnArgs &a);
// CTAs a launch_gemm of this shape and configuration runs.
uint32_t gemm_ctas(uint32_t m, uint32_t n, const GemmConfig &cfg);
size_t attn_counters(uint32_t n, uint32_t heads);
bool launch_attention(const AttnArgs &a, cudaStream_t s, bool pdl);
uint32_t choose_kv_chunks(uint32_t n, uint32_t heads, uint32_t window, int sms, bool packed = false);
// The shortest global / sliding-window sequences for the tensor-core attention: sets both,
// returns the old values in place.
void swap_attn_tc_min(uint32_t *global_min, uint32_t *window_min);

// ---------------------------------------------------------------------------------------------
// memory-bound edges

bool launch_embed(const uint32_t *ids, uint32_t n, const __half *table, const float *gamma,
                  uint32_t d, float eps, __half *x, float *stats, cudaStream_t s, bool pdl);
bool launch_norm_add(const __half *x, uint32_t n, uint32_t d, const float *gamma,
                     const float *add, float eps, __half *out, float *stats, cudaStream_t s,
                     bool pdl);
bool launch_score(const __half *y, uint32_t d, const __half *w, float b, const uint32_t *markers,
                  uint32_t k, float *logits, cudaStream_t s, bool pdl);
// Gathers the marker rows of x and their statistics (for the scorer, which only needs those).
// A marker >= limit records JC_DEV_BAD_INDEX in `err` (nullptr: the module's word) and is not
// read.
bool launch_gather_rows(const __half *x, const float *stats, uint32_t d, const uint32_t *rows,
                        uint32_t k, uint32_t limit, __half *out, float *out_stats, cudaStream_t s,
                        bool pdl, unsigned int *err);

// Device error words: an engine's own (a device pointer) or, for nullptr, the module's word that
// the per-kernel entry points record into. Reads (and clears, when set) one, synchronously.
bool read_device_error(unsigned int *code, unsigned int *word);
// Queues a copy of an error word into pinned host memory on stream s (read it after the stream
// has synchronised).
bool enqueue_device_error_read(unsigned int *pinned, cudaStream_t s, unsigned int *word);
// Clears an error word (synchronous).
bool clear_device_error(unsigned int *word);
const char *device_error_name(unsigned int code);

// ---------------------------------------------------------------------------------------------
// persistent kernel (persist.cuh): a phase list run by one cooperative launch

struct PhaseDesc;
// Resident CTAs of the persistent kernel per SM (0 on error).
int persist_blocks_per_sm();
// Fills the dataflow schedule of a launch's phases d[0, n) on `grid` CTAs (each GEMM phase's tile
// width, rows, items, first item, dependencies on the phases before it in the same launch;
// PhaseDesc::extra set to 0) and returns the launch's item count. GEMM phases run 64- or
// 32-column tiles (persist_tile_width), so their n is a multiple of 32 (64 for RoPE and GeGLU).
uint32_t plan_flow(PhaseDesc *d, uint32_t n, uint32_t grid);
// The plan's cost model (us, B200): one 128-row tile of width bn over depth k, a phase of m x n x
// k on `grid` CTAs, and the persistent kernel's tile width for a GEMM phase.
double gemm_tile_us(uint32_t k, int bn);
double gemm_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid);
double persist_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid);
uint32_t persist_tile_width(uint32_t m, uint32_t n, uint32_t k, uint32_t epi, uint32_t grid);
// The persistent kernel's tile width policy (0 the plan, 64 or 32): sets it, returns the old one.
void swap_persist_tile_policy(int *bn);
// Counter words a launch of n_phases phases over `blocks` 128-row blocks needs (zeroed once; the
// kernel leaves them zero).
inline size_t flow_counter_words(uint32_t n_phases, uint32_t blocks) {
    return (size_t)n_phases * blocks + 3;
}
// phases: device copies of plan_flow's output; timeout_ns: how long a dependency wait may last;
// err: the error word a timeout is recorded in (nullptr: the module's).
bool launch_persist(const PhaseDesc *phases, uint32_t n_phases, uint32_t total_items, uint32_t *ctr,
                    uint32_t blocks, uint32_t grid, uint64_t timeout_ns, cudaStream_t s,
                    unsigned int *err, uint64_t *prof = nullptr, uint32_t prof_cap = 0);

}  // namespace jc
