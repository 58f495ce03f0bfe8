// jc_gemm_noalloc: the fused-epilogue GEMM (jc_gemm) for callers that cannot allocate device
// memory, e.g. a serving loop whose memory was planned up front, or code that runs where a
// cudaMalloc would synchronise the device or fail. Its split-K scratch (the f32 partial tiles and
// the per-tile arrival counters that jc_gemm otherwise takes from the caller) lives in fixed arrays
// of this library's device memory instead, so the caller passes only inputs and outputs.
//
// The arrays are file-scope device variables: every GPU that loads the library holds them
// (JC_NOALLOC_WS_FLOATS floats + JC_NOALLOC_COUNTERS counters, 16 MiB + 16 KiB) until the process
// exits. In host code their names are host-side stand-ins, not device addresses, so their device
// addresses are looked up with cudaGetSymbolAddress once per device (with that device current) on
// the first call there, and that address is what the kernel receives.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "jc_internal.h"

#define JC_NOALLOC_WS_FLOATS (4u << 20)
#define JC_NOALLOC_COUNTERS 4096u

static __device__ __align__(256) float g_noalloc_ws[JC_NOALLOC_WS_FLOATS];
static __device__ __align__(256) uint32_t g_noalloc_counters[JC_NOALLOC_COUNTERS];

namespace {

struct DeviceScratch {
    float *ws = nullptr;
    uint32_t *counters = nullptr;
};

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
DeviceScratch g_scratch[kMaxDevices];

// The device addresses of the arrays on the current device (looked up on its first use).
bool scratch_for_current_device(DeviceScratch *out) {
    int dev = 0;
    if (!jc::cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return false;
    if (dev < 0 || dev >= kMaxDevices) {
        jc::set_error("gemm_noalloc: device index out of range");
        return false;
    }
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceScratch &s = g_scratch[dev];
    if (!s.ws) {
        void *ws = nullptr, *cnt = nullptr;
        if (!jc::cuda_ok(cudaGetSymbolAddress(&ws, g_noalloc_ws), "cudaGetSymbolAddress") ||
            !jc::cuda_ok(cudaGetSymbolAddress(&cnt, g_noalloc_counters), "cudaGetSymbolAddress"))
            return false;
        s.ws = static_cast<float *>(ws);
        s.counters = static_cast<uint32_t *>(cnt);
    }
    *out = s;
    return true;
}

}  // namespace

extern "C" int jc_gemm_noalloc(uint32_t epi, int bn, int splits, const uint16_t *a,
                               const uint16_t *w, uint16_t *c, const uint16_t *res,
                               const float *stats_in, const float *colsum, float *stats_out,
                               float *zero, uint32_t zero_len, uint32_t m, uint32_t n, uint32_t k,
                               float eps, const float *rope, const float *bias, void *stream) {
    try {
        if (!a || !w) {
            jc::set_error("gemm_noalloc: null a or w");
            return -1;
        }
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        jc::GemmConfig cfg = jc::choose_gemm(m, n, k, sms);
        if ((epi & (JC_EPI_ROPE | JC_EPI_GEGLU)) && cfg.bn < 64) cfg.bn = 64;
        if (bn) cfg.bn = bn;
        jc::request_splits(cfg, splits);
        jc::set_gemm_depth(cfg, m, n, sms);
        if (cfg.bn <= 0 || n % cfg.bn) {
            jc::set_error("gemm_noalloc: n must be a multiple of the tile width");
            return -1;
        }
        // An automatic choice (splits = 0) that would need more scratch than the fixed array
        // holds takes fewer workspace splits instead of being refused; an explicit request is
        // honoured or refused below.
        while (splits == 0 && cfg.splits > 1 &&
               (jc::gemm_ws_floats(m, n, cfg) > JC_NOALLOC_WS_FLOATS ||
                jc::gemm_counters(m, n, cfg) > JC_NOALLOC_COUNTERS)) {
            cfg.splits--;
            jc::set_gemm_depth(cfg, m, n, sms);
        }
        const size_t ws_need = jc::gemm_ws_floats(m, n, cfg);
        const size_t cnt_need = jc::gemm_counters(m, n, cfg);
        if (ws_need > JC_NOALLOC_WS_FLOATS || cnt_need > JC_NOALLOC_COUNTERS) {
            jc::set_error("gemm_noalloc: this shape and split-K need " + std::to_string(ws_need) +
                          " scratch floats and " + std::to_string(cnt_need) +
                          " counters; the fixed scratch holds " +
                          std::to_string(JC_NOALLOC_WS_FLOATS) + " and " +
                          std::to_string(JC_NOALLOC_COUNTERS) + " (use fewer splits, or jc_gemm)");
            return -1;
        }
        DeviceScratch sc;
        if (!scratch_for_current_device(&sc)) return -1;
        jc::GemmArgs g;
        g.epi = epi;
        g.c = reinterpret_cast<__half *>(c);
        g.res = reinterpret_cast<const __half *>(res);
        g.ws = sc.ws;
        g.counters = sc.counters;
        g.stats_in = stats_in;
        g.colsum = colsum;
        g.stats_out = stats_out;
        g.zero = zero;
        g.zero_len = zero_len;
        g.m = m;
        g.n = n;
        g.k = k;
        g.eps = eps;
        g.rope = rope;
        g.bias = bias;
        if (!jc::check_gemm(g, cfg) || !jc::make_tmap_f16(&g.map_a, a, m, k, (uint32_t)cfg.bm) ||
            !jc::make_tmap_f16(&g.map_w, w, n, k, jc::gemm_w_rows(cfg)))
            return -1;
        // The counters start every call at zero: a call that stopped early (a device-side
        // timeout) could have left some behind.
        if (cnt_need && !jc::cuda_ok(cudaMemsetAsync(sc.counters, 0, cnt_need * sizeof(uint32_t),
                                                     (cudaStream_t)stream),
                                     "clear counters"))
            return -1;
        return jc::launch_gemm(g, cfg, (cudaStream_t)stream, true) ? 0 : -1;
    } catch (...) {
        jc::set_error("gemm_noalloc: unexpected exception");
        return -1;
    }
}
