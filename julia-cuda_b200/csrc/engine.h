// Engine: one model on one GPU with every buffer a request needs preallocated for max_length
// tokens, the forward pass as a chain of launches (or one persistent launch per layer), captured
// into CUDA graphs per request shape. The reference's Engine / GpuEncoder / GpuHead
// (src/engine.rs, src/forward.rs), re-planned for the B200.
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

namespace jc {

struct GraphKey {
    uint32_t n, k, qtype;
    int fused;
    bool operator==(const GraphKey &o) const {
        return n == o.n && k == o.k && qtype == o.qtype && fused == o.fused;
    }
    bool operator<(const GraphKey &o) const {
        return std::tie(n, k, qtype, fused) < std::tie(o.n, o.k, o.qtype, o.fused);
    }
};

class Engine {
   public:
    static Engine *create(const jc_model_config &cfg, const float *raw, size_t max_length,
                          int device, std::string *why);
    ~Engine();

    // Queues one sequence whose ids / markers are already in the engine's buffers.
    bool enqueue_forward(uint32_t n, uint32_t k, uint32_t qtype, int fused, uint16_t *d_trace,
                         cudaStream_t s);
    // Same, through a cached CUDA graph of that shape.
    bool launch_forward(uint32_t n, uint32_t k, uint32_t qtype, int fused, cudaStream_t s);
    int launches_per_forward(uint32_t n, uint32_t k, int fused) const;
    bool check_device_error(std::string *why);

    jc_model_config cfg{};
    int device = 0, sms = 0;
    size_t max_length = 0;
    std::string name;
    cudaStream_t stream = nullptr;

    // inputs / outputs of one request (device)
    uint32_t *ids = nullptr, *markers = nullptr, *iota = nullptr;
    float *logits = nullptr;
    // pinned staging for julia_cuda_run
    static constexpr int QUEUE = 16;
    uint32_t *h_ids = nullptr, *h_markers = nullptr;  // QUEUE slots of max_length
    float *h_logits = nullptr;
    cudaEvent_t ev_start[QUEUE] = {}, ev_end[QUEUE] = {};

   private:
    Engine() = default;
    bool init(const float *raw, std::string *why);
    const CUtensorMap *wmap(const void *p, uint32_t rows, uint32_t cols, int bn);
    bool gemm(uint32_t epi, const CUtensorMap &amap, const void *w, uint32_t m, uint32_t n,
              uint32_t k, __half *c, const __half *res, const float *stats_in,
              const float *colsum, float *stats_out, float *zero, uint32_t zero_len,
              const float *rope, const float *bias, float eps, cudaStream_t s);
    bool attention(const __half *qkv, __half *o, uint32_t n, uint32_t window, cudaStream_t s);
    bool encoder_layer(int l, uint32_t n, cudaStream_t s);
    bool head_and_scorer(uint32_t n, uint32_t k, uint32_t qtype, cudaStream_t s);

    HostWeights hw;  // layout only after upload (arenas freed)
    uint16_t *w16 = nullptr;
    float *w32 = nullptr;
    __half *x = nullptr, *qkv = nullptr, *o = nullptr, *mb = nullptr, *hx = nullptr,
           *xs = nullptr, *ys = nullptr;
    float *stats_a = nullptr, *stats_b = nullptr, *stats_s = nullptr;
    float *gemm_ws = nullptr, *attn_ws = nullptr;
    uint32_t *gemm_cnt = nullptr, *attn_cnt = nullptr;
    size_t gemm_ws_cap = 0, gemm_cnt_cap = 0, attn_ws_cap = 0, attn_cnt_cap = 0;
    CUtensorMap tm_x{}, tm_o{}, tm_m{}, tm_f{}, tm_hx{}, tm_xs{};
    std::map<std::tuple<const void *, uint32_t, uint32_t, int>, CUtensorMap> wmaps;
    std::map<GraphKey, cudaGraphExec_t> graphs;
    std::list<GraphKey> graph_lru;
    std::vector<void *> allocations;
};

}  // namespace jc
