// Engine: one model on one GPU with every buffer a request needs preallocated for max_length
// tokens. The forward pass is a list of steps (GEMMs with fused epilogues, attention, row-wise
// edges) that runs either as one kernel per step, as one persistent launch per encoder layer, or
// as a single persistent launch for the whole model; each request shape is captured once into a
// CUDA graph. The reference's Engine / GpuEncoder / GpuHead (src/engine.rs, src/forward.rs),
// re-planned for the B200.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <list>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "jc_internal.h"
#include "model.h"
#include "params.h"

namespace jc {

// Execution modes (the C ABI's layer_fused argument).
enum : int { MODE_STEPS = 0, MODE_LAYER = 1, MODE_MODEL = 2 };

struct GraphKey {
    uint32_t n, k, qtype;
    int mode;
    uint32_t head;    // rows the head runs on
    uint32_t packed;  // several requests in one forward (their segments in the engine's seg)
    bool operator==(const GraphKey &o) const {
        return n == o.n && k == o.k && qtype == o.qtype && mode == o.mode && head == o.head &&
               packed == o.packed;
    }
    bool operator<(const GraphKey &o) const {
        return std::tie(n, k, qtype, mode, head, packed) <
               std::tie(o.n, o.k, o.qtype, o.mode, o.head, o.packed);
    }
};

// Where a traced forward copies its intermediate results (device, f16; nullptr: not traced):
// enc [n_layers][n][D] the residual stream after each encoder layer; head [n_head_layers + 1][nh]
// [D] the head's stream (its input, then after each head layer; nh = the head's rows); scorer
// [k][scorer_hidden] the scorer's hidden layer (after GELU) of each marker.
// prof: a profiling run's per-CTA phase stamps, prof_cap 8-word records for each launch (launch i
// of the forward writes records [i * prof_cap, (i + 1) * prof_cap)); per-step kernels only.
struct Trace {
    uint16_t *enc = nullptr, *head = nullptr, *scorer = nullptr;
    uint64_t *prof = nullptr;
    uint32_t prof_cap = 0;
};

struct Step {
    PhaseDesc d{};      // device-ready descriptor (tensor-map pointers into the device map array)
    int map_a = -1;     // host copy of the A operand's tensor map (index)
    const void *w = nullptr;  // GEMM weights, for the single-GEMM kernels' own maps
    int layer = -1;     // encoder layer, or -1 before the encoder, -2 after it
    uint32_t flow_total = 0;  // first step of a persistent launch: the launch's work items
    int slot = -1;      // the step's index in its forward (its phase-stamp records, when profiled)
};

class Engine {
   public:
    static Engine *create(const jc_model_config &cfg, const float *raw, size_t max_length,
                          int device, std::string *why);
    ~Engine();

    // Queues one sequence whose ids / markers are already in the engine's buffers.
    bool enqueue_forward(uint32_t n, uint32_t k, uint32_t qtype, int mode, const Trace &tr,
                         cudaStream_t s);
    // Same, through a cached CUDA graph of that shape.
    // packed: the n rows hold several requests (rows [seg[r].x, seg[r].y) per row r of the
    // device array `seg`); attention stays within a request and RoPE positions restart.
    bool launch_forward(uint32_t n, uint32_t k, uint32_t qtype, int mode, cudaStream_t s,
                        bool packed = false);
    int launches_per_forward(uint32_t n, uint32_t k, int mode) const;
    // Reads (and clears) this engine's device error word; on an error also resets every counter
    // its kernels keep (persistent-kernel dependencies, split-K and split-KV arrivals), since a
    // wait that gave up can leave them mid-way.
    bool check_device_error(std::string *why);
    // The same, returning the code (0: none) instead of a message.
    bool take_device_error(unsigned int *code);
    // Runs the persistent kernel with a grid barrier that waits for one CTA too many, so it must
    // time out after timeout_ns; returns the device error code it recorded.
    bool barrier_timeout_probe(uint64_t timeout_ns, uint32_t *code);

    jc_model_config cfg{};
    int device = 0, sms = 0;
    uint32_t persist_grid = 0;
    size_t max_length = 0;
    std::string name;
    cudaStream_t stream = nullptr;
    uint64_t barrier_timeout_ns = 2000000000ull;
    // The head (final LayerNorm, head layers, marker gather) runs on rows [0, head_length) of a
    // longer sequence; 0 = every row (the reference's GPU head). Markers must lie inside.
    size_t head_length = 0;
    // julia_cuda_run packs consecutive requests (same question type, no head length) into
    // forwards of up to pack_rows tokens; 0 = one forward per request (the reference's way).
    size_t pack_rows = 0;
    uint32_t head_rows(uint32_t n) const {
        return head_length && head_length < n ? (uint32_t)head_length : n;
    }

    // inputs / outputs of one forward (device): ids at [0, L), markers at [L, 2L) and, for
    // packed requests, each row's request rows (uint2) at [2L, 4L) of one allocation
    uint32_t *ids = nullptr, *markers = nullptr, *iota = nullptr;
    uint2 *seg = nullptr;
    // packed forwards: the tcgen05 attention's request-aligned tiles, at [4L, 4L + 2 cap) of the
    // same allocation (cap = attn_tile_cap(L) entries)
    uint2 *tiles = nullptr;
    // Words of a forward's inputs (ids, markers, segments, tiles), on the device and in each
    // staging slot.
    size_t input_words() const { return 4 * (size_t)max_length + 2 * (size_t)attn_tile_cap((uint32_t)max_length); }
    float *logits = nullptr;
    // pinned staging for julia_cuda_run
    static constexpr int QUEUE = 16;
    // QUEUE slots of 4 x max_length words: the ids, the markers, the segments (the device buffers
    // are one allocation in the same layout, so a forward's inputs are one copy)
    uint32_t *h_ids = nullptr;
    float *h_logits = nullptr;
    unsigned int *h_err = nullptr;  // the device error word, copied after each queue of requests
    // The engine's own device error word: every kernel it launches records device-side timeouts
    // here (not in the module's word, which bare jc_* calls use), so engines sharing a GPU never
    // see or clear each other's errors.
    unsigned int *dev_err = nullptr;
    // The error word copied into h_err (the stream has synchronised since): 0, or the reason.
    bool check_device_error_copy(std::string *why);
    cudaEvent_t ev_start[QUEUE] = {}, ev_end[QUEUE] = {};
    // While set, every launch appends what it ran, a persistent launch one entry per phase (a
    // profiling run's launch list).
    std::vector<jc_launch_info> *launch_log = nullptr;

   private:
    struct GraphEntry {
        cudaGraphExec_t exec = nullptr;
        void *descs = nullptr;
        std::list<GraphKey>::iterator lru;  // this key's place in graph_lru
    };
    Engine() = default;
    bool init(const float *raw, std::string *why);
    int add_map(const void *p, uint32_t rows, uint32_t cols, uint32_t box);
    const CUtensorMap *wmap(const void *p, uint32_t rows, uint32_t cols, int bn);
    // Fills the persistent kernel's schedule of each launch the mode makes (the whole list, or
    // each encoder layer's steps) and the launches' item counts.
    // Each GEMM phase's weights map matches the tile width the plan chose; false (error set) if
    // the engine holds no such map.
    bool plan_steps(std::vector<Step> &steps, int mode) const;
    std::vector<Step> build_steps(uint32_t n, uint32_t k, uint32_t qtype, const Trace &tr,
                                  int mode, bool packed = false) const;
    std::vector<Step> build_steps_flat(uint32_t n, uint32_t k, uint32_t qtype, const Trace &tr,
                                       int mode) const;
    Step gemm_step(uint32_t epi, int map_a, int map_w, const void *w, uint32_t m, uint32_t n,
                   uint32_t k, __half *c, const __half *res, const float *stats_in,
                   const float *colsum, float *stats_out, float *zero, uint32_t zero_len,
                   const float *rope, const float *bias, float eps, int layer) const;
    bool run_step(const Step &st, cudaStream_t s);
    // prof / prof_cap: a profiling run's records (prof_cap per step; a persistent launch of steps
    // [i, j) records its items in the (j - i) x prof_cap records from step i's).
    bool enqueue_steps(const std::vector<Step> &steps, int mode, const PhaseDesc *descs,
                       uint16_t *d_trace, uint32_t n, cudaStream_t s, uint64_t *prof = nullptr,
                       uint32_t prof_cap = 0);
    // A profiling run: appends one entry per phase of a persistent launch of steps [i, j).
    void log_persist(const std::vector<Step> &steps, size_t i, size_t j, uint32_t prof_cap);
    // After a device error: clears the error word and every counter a wait that gave up may have
    // left non-zero (synchronous).
    bool reset_after_error();

    HostWeights hw;  // layout only after upload (arenas freed)
    uint16_t *w16 = nullptr;
    float *w32 = nullptr;
    // RoPE tables in the GEMM epilogue's layout (global, then local), rope_rows positions each
    float *rope_t = nullptr;
    uint32_t rope_rows = 0;
    __half *x = nullptr, *qkv = nullptr, *o = nullptr, *mb = nullptr, *hx = nullptr,
           *xs = nullptr, *ys = nullptr;
    float *stats_a = nullptr, *stats_b = nullptr, *stats_s = nullptr;
    float *gemm_ws = nullptr, *attn_ws = nullptr;
    uint32_t *gemm_cnt = nullptr, *attn_cnt = nullptr;
    // the persistent kernel's completion / work counters (scratch_cap phases x flow_blocks + 3)
    uint32_t *flow_ctr = nullptr;
    uint32_t flow_blocks = 0;
    size_t gemm_ws_cap = 0, gemm_cnt_cap = 0, attn_ws_cap = 0, attn_cnt_cap = 0;
    // tensor maps: host copies and the device array the persistent kernel reads
    std::vector<CUtensorMap> hmaps;
    // what each of hmaps covers (an A operand's map for another tile height is derived from it)
    struct MapSrc {
        const void *p;
        uint32_t rows, cols;
    };
    std::vector<MapSrc> map_src;
    std::map<std::tuple<const void *, uint32_t, uint32_t, uint32_t>, int> map_index;
    CUtensorMap *dmaps = nullptr;
    int m_x = -1, m_o = -1, m_m = -1, m_f = -1, m_hx = -1, m_xs = -1;
    struct LayerMaps {
        int wqkv, wo, wi, wo_mlp;
    };
    std::vector<LayerMaps> lmaps;
    struct HeadMaps {
        int in, out, l1, l2;
    };
    std::vector<HeadMaps> hmaps_head;
    int m_s1 = -1;
    // descriptors for launches outside a graph (one forward's worth)
    PhaseDesc *scratch_descs = nullptr;
    size_t scratch_cap = 0;
    std::map<std::tuple<const void *, uint32_t, uint32_t, int>, CUtensorMap> wmaps;
    std::map<GraphKey, GraphEntry> graphs;
    std::list<GraphKey> graph_lru;
    std::vector<void *> allocations;
};

}  // namespace jc
