// The library's only CUDA translation unit: every kernel template is instantiated here, next to
// its host launcher (argument checks, launch shape, PDL attribute). Keeping one unit lets all
// kernels share the device error word without relocatable device code.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "attention_tc.cuh"
#include "edges.cuh"
#include "gemm.cuh"
#include "gemm_pair.cuh"
#include "gemm_persist.cuh"
#include "jc_internal.h"
#include "persist.cuh"

namespace jc {

static thread_local std::string t_error;
void set_error(const std::string &msg) { t_error = msg; }
const char *last_error() { return t_error.c_str(); }

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

bool read_device_error(unsigned int *code, unsigned int *word) {
    if (word) {
        if (!cuda_ok(cudaMemcpy(code, word, sizeof(unsigned int), cudaMemcpyDeviceToHost),
                     "read error word"))
            return false;
        return *code == 0 || clear_device_error(word);
    }
    if (!cuda_ok(cudaMemcpyFromSymbol(code, g_dev_error, sizeof(unsigned int)), "read error word"))
        return false;
    return *code == 0 || clear_device_error(nullptr);
}

bool enqueue_device_error_read(unsigned int *pinned, cudaStream_t s, unsigned int *word) {
    if (word)
        return cuda_ok(cudaMemcpyAsync(pinned, word, sizeof(unsigned int), cudaMemcpyDeviceToHost, s),
                       "read error word");
    return cuda_ok(cudaMemcpyFromSymbolAsync(pinned, g_dev_error, sizeof(unsigned int), 0,
                                             cudaMemcpyDeviceToHost, s),
                   "read error word");
}

bool clear_device_error(unsigned int *word) {
    unsigned int zero = 0;
    if (word)
        return cuda_ok(cudaMemcpy(word, &zero, sizeof(zero), cudaMemcpyHostToDevice), "clear error word");
    return cuda_ok(cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero)), "clear error word");
}

const char *device_error_name(unsigned int code) {
    switch (code) {
        case 0: return "none";
        case JC_DEV_TIMEOUT_FULL: return "a GEMM operand stage never arrived (TMA wait timed out)";
        case JC_DEV_TIMEOUT_EMPTY: return "a GEMM stage was never released (MMA wait timed out)";
        case JC_DEV_TIMEOUT_MMA: return "a GEMM accumulator was never committed (wait timed out)";
        case JC_DEV_TIMEOUT_GRID: return "a grid barrier timed out";
        case JC_DEV_TIMEOUT_SPLIT: return "split partials never completed (wait timed out)";
        case JC_DEV_BAD_INDEX: return "an index checked on the device was out of range";
        default: return "unknown device error";
    }
}

// ---------------------------------------------------------------------------------------------
// launch helper: cudaLaunchKernelEx with programmatic stream serialization when `pdl`

static uint32_t env_u32_early(const char *name, uint32_t dflt) {
    const char *e = getenv(name);
    return e ? (uint32_t)strtoul(e, nullptr, 10) : dflt;
}

// Programmatic dependent launch is on unless the environment sets JC_PDL=0 (for A/B timing).
static bool pdl_allowed() {
    static const bool on = [] {
        const char *v = getenv("JC_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
static bool launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      bool pdl, const char *what, Args... args) {
    pdl = pdl && pdl_allowed();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cuda_ok(cudaLaunchKernelEx(&cfg, kern, args...), what);
}

// launch_ex with the grid grouped into thread-block clusters of `cluster_z` CTAs along z (1: none).
template <typename... KArgs, typename... Args>
static bool launch_ex_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, bool pdl, int cluster_z, const char *what,
                              Args... args) {
    pdl = pdl && pdl_allowed();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    if (cluster_z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = 1;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = (unsigned)cluster_z;
        n++;
    }
    cfg.attrs = n ? attr : nullptr;
    cfg.numAttrs = n;
    return cuda_ok(cudaLaunchKernelEx(&cfg, kern, args...), what);
}

// Sets a kernel's dynamic shared-memory limit once per device.
template <typename K>
static bool ensure_smem(K kern, int bytes, std::atomic<uint64_t> &done_mask) {
    int dev = 0;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return false;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load() & bit) return true;
    if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                 "cudaFuncSetAttribute"))
        return false;
    done_mask.fetch_or(bit);
    return true;
}

// ---------------------------------------------------------------------------------------------
// TMA descriptors

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

bool make_tmap_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                   uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
        return false;
    }
    if (cols % 64) {
        set_error("a GEMM operand's columns must be a multiple of 64");
        return false;
    }
    // dims: 64 columns of a k-block, rows, k-blocks; strides (bytes): a row, a k-block (128 B).
    cuuint64_t dims[3] = {64, rows, cols / 64};
    cuuint64_t strides[2] = {cols * 2, 128};
    cuuint32_t box[3] = {64, box_rows, (cuuint32_t)GEMM_KPS};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides,
                    box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
        return false;
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// GEMM

size_t gemm_ws_floats(uint32_t m, uint32_t n, GemmConfig cfg) {
    if (cfg.splits <= 1) return 0;
    const size_t tiles = (size_t)((m + cfg.bm - 1) / cfg.bm) * (n / cfg.bn);
    return tiles * cfg.splits * cfg.bn * cfg.bm;
}

size_t gemm_counters(uint32_t m, uint32_t n, GemmConfig cfg) {
    if (cfg.splits <= 1) return 0;
    return (size_t)((m + cfg.bm - 1) / cfg.bm) * (n / cfg.bn);
}

// Stage depths: "shallow" keeps a CTA near 100 KB of shared memory so two fit on an SM (a GEMM
// and the next kernel's early CTAs under PDL); "deep" doubles the bytes in flight per CTA for
// grids of at most one CTA per SM, where one CTA's pipeline latency bounds the kernel.
template <int BN> struct Depth;
template <> struct Depth<32> { static constexpr int shallow = 2, deep = 5; };
template <> struct Depth<64> { static constexpr int shallow = 2, deep = 4; };
template <> struct Depth<128> { static constexpr int shallow = 2, deep = 3; };
template <> struct Depth<256> { static constexpr int shallow = 2, deep = 2; };  // 96 KB stages
// 64-row tiles (one CTA per SM): a stage holds half the activation bytes, so the ring goes deeper
// and holds a whole 1152-deep K range of a 32-column tile (9 stages would; 8 x 24 KB fit).
// Cluster split-K: each CTA's K range is 1/CS of the whole, so a short ring holds it (3 stages of a
// 64-column tile cover K = 768 / 2), beside the receive buffer of the peers' partials.
template <int BN> struct DepthCluster;
template <> struct DepthCluster<64> { static constexpr int stages = 3; };
template <> struct DepthCluster<128> { static constexpr int stages = 2; };
template <int BN> struct Depth64;
template <> struct Depth64<32> { static constexpr int shallow = 4, deep = 8; };  // 24 KB stages
template <> struct Depth64<64> { static constexpr int shallow = 3, deep = 6; };  // 32 KB stages

template <int BN, int STAGES, uint32_t EPI, int CS, int BM>
static bool launch_gemm_inst(const GemmKernelParams &p, dim3 grid, cudaStream_t s, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    auto kern = gemm_tc_kernel<BN, STAGES, EPI, CS, BM>;
    using Sh = GemmShape<BN, STAGES, BM>;
    constexpr int smem = Sh::SMEM_BYTES + Sh::template RECV_BYTES<CS>;
    static_assert(smem <= 227 * 1024, "a GEMM CTA's shared memory");
    if (!ensure_smem(kern, smem, smem_set)) return false;
    return launch_ex_cluster(kern, grid, dim3(GEMM_THREADS), smem, s, pdl, CS, "gemm launch", p);
}

template <int BN, int STAGES, int CS, int BM = GEMM_BM>
static bool launch_gemm_depth(uint32_t epi, const GemmKernelParams &p, dim3 grid, cudaStream_t s,
                              bool pdl) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    switch (epi) {
        case 0: return launch_gemm_inst<BN, STAGES, 0, CS, BM>(p, grid, s, pdl);
        case RS: return launch_gemm_inst<BN, STAGES, RS, CS, BM>(p, grid, s, pdl);
        case JC_EPI_BIAS | RS: return launch_gemm_inst<BN, STAGES, JC_EPI_BIAS | RS, CS, BM>(p, grid, s, pdl);
        case LB: return launch_gemm_inst<BN, STAGES, LB, CS, BM>(p, grid, s, pdl);
        case LB | JC_EPI_RELU: return launch_gemm_inst<BN, STAGES, LB | JC_EPI_RELU, CS, BM>(p, grid, s, pdl);
        case LB | JC_EPI_GELU: return launch_gemm_inst<BN, STAGES, LB | JC_EPI_GELU, CS, BM>(p, grid, s, pdl);
        default: break;
    }
    if constexpr (BN >= 64) {
        switch (epi) {
            case JC_EPI_ROPE: return launch_gemm_inst<BN, STAGES, JC_EPI_ROPE, CS, BM>(p, grid, s, pdl);
            case JC_EPI_LN | JC_EPI_ROPE:
                return launch_gemm_inst<BN, STAGES, JC_EPI_LN | JC_EPI_ROPE, CS, BM>(p, grid, s, pdl);
            case JC_EPI_LN | JC_EPI_GEGLU:
                return launch_gemm_inst<BN, STAGES, JC_EPI_LN | JC_EPI_GEGLU, CS, BM>(p, grid, s, pdl);
            default: break;
        }
    }
    set_error("gemm: no kernel for epilogue " + std::to_string(epi) + " with " +
              std::to_string(BN) + "-column tiles");
    return false;
}

template <int BN>
static bool launch_gemm_bn(uint32_t epi, const GemmConfig &cfg, const GemmKernelParams &p,
                           dim3 grid, cudaStream_t s, bool pdl) {
    if constexpr (BN <= 64) {
        if (cfg.bm == 64)
            return cfg.deep ? launch_gemm_depth<BN, Depth64<BN>::deep, 1, 64>(epi, p, grid, s, pdl)
                            : launch_gemm_depth<BN, Depth64<BN>::shallow, 1, 64>(epi, p, grid, s, pdl);
    }
    // Cluster split-K runs with the shallow ring: a cluster's CTAs share the tile's K loop.
    if constexpr (BN >= 64 && BN <= 128) {
        if (cfg.cluster == 2) return launch_gemm_depth<BN, DepthCluster<BN>::stages, 2>(epi, p, grid, s, pdl);
        if (cfg.cluster == 4) return launch_gemm_depth<BN, DepthCluster<BN>::stages, 4>(epi, p, grid, s, pdl);
    }
    return cfg.deep ? launch_gemm_depth<BN, Depth<BN>::deep, 1>(epi, p, grid, s, pdl)
                    : launch_gemm_depth<BN, Depth<BN>::shallow, 1>(epi, p, grid, s, pdl);
}

template <int BN, int STAGES>
static bool launch_gemm_persist(uint32_t epi, const GemmKernelParams &p, dim3 grid, cudaStream_t s,
                                bool pdl) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    constexpr int smem = GemmPersistShape<BN, STAGES>::SMEM_BYTES + 1024;
    auto go = [&](auto kern, std::atomic<uint64_t> &set) {
        if (!ensure_smem(kern, smem, set)) return false;
        return launch_ex(kern, grid, dim3(PERSIST_GEMM_THREADS), smem, s, pdl, "gemm launch", p);
    };
#define JC_PERSIST(E)                                                   \
    case E: {                                                           \
        static std::atomic<uint64_t> set{0};                            \
        return go(gemm_persistent_kernel<BN, STAGES, E>, set);          \
    }
    switch (epi) {
        JC_PERSIST(0)
        JC_PERSIST(RS)
        JC_PERSIST(JC_EPI_BIAS | RS)
        JC_PERSIST(LB)
        JC_PERSIST(LB | JC_EPI_RELU)
        JC_PERSIST(LB | JC_EPI_GELU)
        JC_PERSIST(JC_EPI_ROPE)
        JC_PERSIST(JC_EPI_LN | JC_EPI_ROPE)
        JC_PERSIST(JC_EPI_LN | JC_EPI_GEGLU)
        default: break;
    }
#undef JC_PERSIST
    set_error("gemm: no compiled kernel for epilogue " + std::to_string(epi));
    return false;
}

// The CTA-pair kernel (gemm_pair.cuh): clusters of two CTAs along x, as many pairs as the tiles
// need and the GPU holds at once (cudaOccupancyMaxActiveClusters, cached per device).
template <int BN, int STAGES>
static bool launch_gemm_pair(uint32_t epi, const GemmKernelParams &p, uint32_t tiles, cudaStream_t s,
                             bool pdl) {
    constexpr uint32_t RS = JC_EPI_RES | JC_EPI_STATS, LB = JC_EPI_LN | JC_EPI_BIAS;
    constexpr int smem = GemmPairShape<BN, STAGES>::SMEM_BYTES + 1024;
    auto go = [&](auto kern, std::atomic<uint64_t> &set, std::atomic<int> &max_pairs) {
        if (!ensure_smem(kern, smem, set)) return false;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(PERSIST_GEMM_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (max_pairs.load() <= 0) {
            int dev = 0, sms = 0, n = 0;
            if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice") ||
                !cuda_ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "sm count"))
                return false;
            cfg.gridDim = dim3(2 * (sms / 2));
            if (!cuda_ok(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "cluster occupancy")) return false;
            if (n <= 0) {
                set_error("gemm: no CTA pair of the pair kernel fits an SM pair");
                return false;
            }
            max_pairs.store(n);
        }
        cfg.gridDim = dim3(2 * std::min<uint32_t>(tiles, (uint32_t)max_pairs.load()));
        if (pdl && pdl_allowed()) {
            attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.numAttrs = 2;
        }
        return cuda_ok(cudaLaunchKernelEx(&cfg, kern, p), "gemm pair launch");
    };
#define JC_PAIR(E)                                                      \
    case E: {                                                           \
        static std::atomic<uint64_t> set{0};                            \
        static std::atomic<int> max_pairs{0};                           \
        return go(gemm_pair_kernel<BN, STAGES, E>, set, max_pairs);     \
    }
    switch (epi) {
        JC_PAIR(0)
        JC_PAIR(RS)
        JC_PAIR(JC_EPI_BIAS | RS)
        JC_PAIR(LB)
        JC_PAIR(LB | JC_EPI_RELU)
        JC_PAIR(LB | JC_EPI_GELU)
        JC_PAIR(JC_EPI_ROPE)
        JC_PAIR(JC_EPI_LN | JC_EPI_ROPE)
        JC_PAIR(JC_EPI_LN | JC_EPI_GEGLU)
        default: break;
    }
#undef JC_PAIR
    set_error("gemm: no compiled pair kernel for epilogue " + std::to_string(epi));
    return false;
}

bool launch_gemm(const GemmArgs &g, GemmConfig cfg, cudaStream_t s, bool pdl) {
    if (!check_gemm(g, cfg)) return false;
    GemmKernelParams kp;
    kp.map_a = g.map_a;
    kp.map_w = g.map_w;
    GemmParams &p = kp.p;
    p.map_a = nullptr;  // the kernel points these at its own copies
    p.map_w = nullptr;
    p.map_c = nullptr;
    p.store_tma = 0;
    // A/B knob JC_GEMM_STORE_TMA=0|1: the staged output tile written by TMA stores (1) or by
    // every thread's coalesced 16-byte stores (0).
    static const uint32_t store_tma = env_u32_early("JC_GEMM_STORE_TMA", 1u);
    if (cfg.cluster == 1 && store_tma) {
        // The output through TMA stores: c as (columns, m rows), boxes of up to 64 columns x 128
        // rows with the swizzle the epilogue stages in; rows past m are not written.
        const bool geglu = g.epi & JC_EPI_GEGLU;
        const uint32_t n_out = geglu ? g.n / 2 : g.n, w_out = geglu ? cfg.bn / 2 : cfg.bn;
        const uint32_t bw = w_out < 64 ? w_out : 64;
        auto fn = encode_fn();
        if (fn && (reinterpret_cast<uintptr_t>(g.c) & 15) == 0 && (n_out * 2) % 16 == 0) {
            cuuint64_t dims[2] = {n_out, g.m};
            cuuint64_t strides[1] = {(cuuint64_t)n_out * 2};
            cuuint32_t box[2] = {bw, (cuuint32_t)cfg.bm};
            cuuint32_t es[2] = {1, 1};
            const CUresult r = fn(&kp.map_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, g.c, dims, strides,
                                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                  bw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            p.store_tma = r == CUDA_SUCCESS ? 1u : 0u;
        }
    }
    p.c = g.c;
    p.res = g.res;
    p.ws = g.ws;
    p.counters = g.counters;
    p.stats_in = g.stats_in;
    p.colsum = g.colsum;
    p.stats_out = g.stats_out;
    p.zero = g.zero;
    p.rope = g.rope;
    p.bias = g.bias;
    p.rope_stride = g.rope_stride ? g.rope_stride : g.m;
    p.seg = g.seg;
    p.zero_len = g.zero_len;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.eps = g.eps;
    p.err = g.err;
    p.prof = g.prof;
    p.prof_cap = g.prof_cap;
    if (cfg.pair) {
        const uint32_t tiles = (g.n / cfg.bn) * ((g.m + 2 * GEMM_BM - 1) / (2 * GEMM_BM));
        kp.p.store_tma = 0;  // stores through the epilogue warps' own buffers
        kp.p.prof = nullptr;  // no phase stamps (a pair walks several tiles)
        return cfg.bn == 128 ? launch_gemm_pair<128, 4>(g.epi, kp, tiles, s, pdl)
                             : launch_gemm_pair<256, 3>(g.epi, kp, tiles, s, pdl);
    }
    if (cfg.persistent && (cfg.bn == 128 || cfg.bn == 256) && cfg.splits == 1 && cfg.cluster == 1) {
        const uint32_t tiles = (g.n / cfg.bn) * ((g.m + GEMM_BM - 1) / GEMM_BM);
        const dim3 pgrid(std::min(tiles, std::max(cfg.grid, 1u)));
        kp.p.store_tma = 0;  // stores through the epilogue warps' own buffers
        kp.p.prof = nullptr;  // no phase stamps (a CTA walks several tiles)
        return cfg.bn == 128 ? launch_gemm_persist<128, 3>(g.epi, kp, pgrid, s, pdl)
                             : launch_gemm_persist<256, 2>(g.epi, kp, pgrid, s, pdl);
    }
    dim3 grid(g.n / cfg.bn, (g.m + cfg.bm - 1) / cfg.bm, cfg.cluster > 1 ? cfg.cluster : cfg.splits);
    switch (cfg.bn) {
        case 32: return launch_gemm_bn<32>(g.epi, cfg, kp, grid, s, pdl);
        case 64: return launch_gemm_bn<64>(g.epi, cfg, kp, grid, s, pdl);
        case 256: return launch_gemm_bn<256>(g.epi, cfg, kp, grid, s, pdl);
        default: return launch_gemm_bn<128>(g.epi, cfg, kp, grid, s, pdl);
    }
}

bool check_gemm(const GemmArgs &g, GemmConfig cfg) {
    const uint32_t e = g.epi;
    const bool ln = e & JC_EPI_LN, res = e & JC_EPI_RES, stats = e & JC_EPI_STATS,
               rope = e & JC_EPI_ROPE, geglu = e & JC_EPI_GEGLU, bias = e & JC_EPI_BIAS;
    auto fail = [](const char *m) { set_error(std::string("gemm: ") + m); return false; };
    if (cfg.bn != 32 && cfg.bn != 64 && cfg.bn != 128 && cfg.bn != 256)
        return fail("tile width must be 32, 64, 128 or 256");
    if (cfg.bm != 128 && cfg.bm != 64) return fail("tile height must be 128 or 64");
    if (cfg.bm == 64 && (cfg.bn > 64 || cfg.splits != 1 || cfg.cluster != 1 || cfg.persistent))
        return fail("64-row tiles are 32 or 64 columns wide, with no split-K");
    if (cfg.pair && (cfg.bn < 128 || cfg.bm != 128 || cfg.splits != 1 || cfg.cluster != 1))
        return fail("CTA-pair tiles are 128 or 256 columns wide (128 rows a CTA), with no split-K");
    if (g.m == 0) return fail("no rows");
    if (g.k == 0 || g.k % GEMM_BK) return fail("k must be a positive multiple of 64");
    if (g.n == 0 || g.n % cfg.bn) return fail("n must be a multiple of the tile width");
    if (cfg.splits < 1 || cfg.splits > 8 || (uint32_t)cfg.splits > g.k / GEMM_BK)
        return fail("split-K must be 1..8 and at most k/64");
    if (cfg.cluster != 1 && cfg.cluster != 2 && cfg.cluster != 4)
        return fail("a split-K cluster must be 1, 2 or 4 CTAs");
    if (cfg.cluster > 1 && (cfg.splits != 1 || cfg.bn < 64 || cfg.bn > 128 || (uint32_t)cfg.cluster > g.k / GEMM_BK))
        return fail("cluster split-K needs 64- or 128-column tiles, no workspace split and k/64 >= cluster");
    if ((rope || geglu) && cfg.bn < 64) return fail("RoPE and GeGLU need 64-column tiles or wider");
    if (rope && g.n % 192) return fail("RoPE needs a qkv output (n a multiple of 3 x 64)");
    if (rope && geglu) return fail("RoPE and GeGLU do not combine");
    if ((res || stats) && geglu) return fail("residual / statistics do not combine with GeGLU");
    if (!g.c) return fail("no output");
    if (ln && (!g.stats_in || !g.colsum)) return fail("the LayerNorm epilogue needs stats_in and colsum");
    if (rope && !g.rope) return fail("the RoPE epilogue needs the (cos, sin) table");
    if (bias && !g.bias) return fail("the bias epilogues need a bias");
    if (res && !g.res) return fail("the residual epilogue needs res");
    if (stats && !g.stats_out) return fail("the statistics epilogue needs stats_out");
    if (g.zero_len && (!g.zero || g.zero == g.stats_in || g.zero == g.stats_out))
        return fail("the buffer to clear must exist and not be one this GEMM reads or adds to");
    if ((reinterpret_cast<uintptr_t>(g.c) | reinterpret_cast<uintptr_t>(g.res) |
         reinterpret_cast<uintptr_t>(g.colsum) | reinterpret_cast<uintptr_t>(g.bias) |
         reinterpret_cast<uintptr_t>(g.rope)) & 15)
        return fail("c, res, colsum, bias and the RoPE table must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(g.stats_in) | reinterpret_cast<uintptr_t>(g.stats_out)) & 7)
        return fail("stats_in and stats_out must be 8-byte aligned");
    if (cfg.splits > 1 && (!g.ws || !g.counters)) return fail("split-K needs a workspace and counters");
    return true;
}

// 128- and 256-column tiles of a launch past one wave run the persistent kernel, unless
// JC_GEMM_PERSIST=0 (an A/B knob) turns it off.
static bool persistent_width(int bn) {
    static const char *persist = getenv("JC_GEMM_PERSIST");
    return (bn == 128 || bn == 256) && !(persist && persist[0] == '0');
}

// CTA-pair policy (gemm_pair.cuh): 1 (every 128- or 256-column unsplit launch), 0 (automatic:
// the launches that would run the single-SM persistent kernel with 256-column tiles), -1
// (never); a tuning and test hook (jc_gemm_pair_policy), JC_GEMM_PAIR sets its start value.
// Measured alone at 6144 rows (us, single-SM persistent against pairs): 2304-wide qkv 29.2 /
// 27.7, wi 30.5 / 29.0 with 256 columns; 128-column pairs lose everywhere (qkv 30.5 / 37.0), and
// below a few thousand rows the single-SM kernels win (qkv at 3072 rows: 18.9 with 128 columns,
// pairs 21.3).
static std::atomic<int> g_pair{(int)env_u32_early("JC_GEMM_PAIR", 0u)};
void swap_gemm_pair_policy(int *policy) { *policy = g_pair.exchange(*policy); }
static bool pair_for(const GemmConfig &c) {
    const int policy = g_pair.load();
    if (policy < 0 || c.bn < 128 || c.bm != 128 || c.splits != 1 || c.cluster != 1) return false;
    return policy == 1 || (c.persistent && c.bn == 256);
}

// Tile height policy: 0 (automatic), 128 (always 128 rows) or 64 (64 rows wherever legal, even
// past one wave); a tuning and test hook (jc_gemm_tile_rows), JC_GEMM_BM sets its start value.
// The default is 128: in the 293-token forward 64-row tiles measured 652.6 against 646.2 us (the
// 768-wide GEMMs alone 6.59 / 7.77 against 6.72 / 7.55 us): a narrow tile's main loop takes
// 160 ns a k-block whatever its operand bytes (or its number of MMA issuer warps).
static std::atomic<int> g_tile_rows{(int)env_u32_early("JC_GEMM_BM", 128u)};
void swap_gemm_tile_rows(int *rows) { *rows = g_tile_rows.exchange(*rows); }

// The tile height for a configuration whose width and split are set, under the automatic policy:
// 64 rows (an M = 64 MMA) when the tile is at most 64 columns wide, unsplit, and the 64-row grid
// still fits one wave, which halves the activation bytes a CTA ingests (a 768-wide GEMM at 293
// tokens: 120 CTAs of 64 x 32 instead of 72 of 128 x 32).
static int pick_bm(uint32_t m, uint32_t n, const GemmConfig &c, int sms) {
    const int policy = g_tile_rows.load();
    if (policy == 128 || c.bn > 64 || c.splits != 1 || c.cluster != 1) return 128;
    const uint64_t ctas64 = (uint64_t)((m + 63) / 64) * (n / c.bn);
    return policy == 64 || ctas64 <= (uint64_t)sms ? 64 : 128;
}

static uint32_t tiles_m_of(uint32_t m) { return (m + GEMM_BM - 1) / GEMM_BM; }

GemmConfig choose_gemm(uint32_t m, uint32_t n, uint32_t k, int sms) {
    GemmConfig c;
    // A CTA's time is a fixed part (set-up, first stage, epilogue, drain: about as long as
    // streaming 256 operand rows) plus its operand stream ((128 + tile width) x k bytes, at what
    // an SM ingests from L2), so a launch takes about waves x (256 + 128 + width): the width with
    // the least of it, ties to the narrower (less epilogue a thread). Up to a wave this is the
    // narrowest tile whose grid fits (measured: 32 columns for the 768-wide GEMMs at 72-293
    // tokens, 64 at 1024; 64 for the 2304-wide ones up to 448 tokens, 128 at 1024); packs of
    // thousands of rows take 256-column tiles (2304-wide at 3072 rows: 25.0 against 26.6 us),
    // which read the activation tile half as often per output column. Past one wave, 128- and
    // 256-column tiles run persistent (gemm_persist.cuh): the fixed part is paid once and each
    // further wave costs about twice its width (measured per extra wave at k = 768: 5.0 us for
    // 128 columns, 9.5 us for 256, against 10.6 / 15.4 us for the first).
    // A single wave of 256-column tiles pays another 256 for its epilogue (128 columns a thread
    // over two accumulators): measured alone, the 768-wide GEMMs at 2048-6144 rows take 17-18.6
    // us as one wave of 256 columns against 11.7-15.0 as 128 (one wave, or persistent), and the
    // 2304-wide ones at 2048 rows 15.3 against 14.7.
    // The tile height for each width (pick_bm) enters the same way: a 64-row tile streams
    // 64 + width operand rows.
    c.bn = 32;
    uint64_t best = ~0ull;
    for (int bn : {32, 64, 128, 256}) {
        if (n % bn) continue;
        GemmConfig t;
        t.bn = bn;
        const int bm = pick_bm(m, n, t, sms);
        const uint64_t ctas = (uint64_t)((m + bm - 1) / bm) * (n / bn);
        const uint64_t waves = (ctas + sms - 1) / sms;
        const uint64_t cost = waves > 1 && bm == 128 && persistent_width(bn)
                                  ? (256 + (uint64_t)bm + bn) + (waves - 1) * 2 * (uint64_t)bn
                                  : waves * (uint64_t)(256 + bm + bn + (bn == 256 ? 256 : 0));
        if (cost < best) {
            best = cost;
            c.bn = bn;
        }
    }
    // Split-K (workspace or cluster) measured slower than one CTA per tile for every encoder
    // shape at 72-1024 tokens (the partial exchange costs more than the shorter K loop saves).
    c.splits = 1;
    // A/B knob JC_GEMM_CLUSTER=2|4: one-wave shapes as cluster split-K (64-column tiles, else
    // 128), each CTA keeping at least two k-blocks.
    static const uint32_t force_cluster = env_u32_early("JC_GEMM_CLUSTER", 0u);
    if (force_cluster == 2 || force_cluster == 4)
        for (int bn : {64, 128})
            if (n % bn == 0 && (uint64_t)tiles_m_of(m) * (n / bn) * force_cluster <= (uint64_t)sms &&
                k / GEMM_BK >= 2 * force_cluster) {
                c.bn = bn;
                c.cluster = (int)force_cluster;
                break;
            }
    set_gemm_depth(c, m, n, sms);
    return c;
}

void request_splits(GemmConfig &c, int splits) {
    if (splits > 0) {
        c.splits = splits;
        c.cluster = 1;
    } else if (splits < 0) {
        c.splits = 1;
        c.cluster = -splits;
    }
}

void set_gemm_depth(GemmConfig &c, uint32_t m, uint32_t n, int sms) {
    c.bm = pick_bm(m, n, c, sms);
    // At most one CTA per SM: the pipeline depth of one CTA bounds the kernel, so go deep.
    const uint32_t ctas = (m + c.bm - 1) / c.bm * (n / c.bn) * c.splits * c.cluster;
    c.deep = ctas <= (uint32_t)sms && c.cluster == 1;
    static const char *force = getenv("JC_GEMM_DEPTH");  // A/B knob: "deep" / "shallow"
    if (force && force[0] == 'd') c.deep = true;
    if (force && force[0] == 's') c.deep = false;
    c.persistent = ctas > (uint32_t)sms && persistent_width(c.bn) && c.splits == 1 && c.cluster == 1 &&
                   c.bm == 128;
    c.pair = pair_for(c);
    c.grid = (uint32_t)sms;
}

// ---------------------------------------------------------------------------------------------
// attention

// Two kernels. The tensor-core kernel (attention_tc.cuh: 128-query CTAs, tcgen05) for global
// attention from ATTN_TC_MIN tokens (its single MMA thread serialises ~130 cycles a
// instruction, so it only pays once the key loop is long; sliding-window layers and shorter
// sequences measured faster on the mma.sync kernel); otherwise the mma.sync kernel with 32-query
// CTAs: 4 key groups from 193 to 384 tokens (256 threads, 132 KB of shared memory), else 2 key
// groups (128 threads, 68 KB: up to three CTAs an SM, spread by spread_smem). Measured alone (cold
// L2, us, global / window), 2 groups against 4 (one CTA an SM: 512 tokens take two waves) and 64 x 2:
// 128 tokens 4.30 / 4.47 (4.76 / 4.97), 293: 6.77 / 5.98 (6.88 / 5.95), 512: 9.85 / 7.17 (13.36 /
// 9.98), 768: 13.04 / 7.54 (64 x 2: 14.08 / 7.32), 1024 window 8.43 (9.35); 64 x 1 and 32 x 1
// were slower throughout. In the 293-token forward 4 groups measured 660.8 against 662.7 us.
// Global attention over exactly five key tiles (257-320 tokens) takes 5 groups of one tile each
// (320 threads, 164 KB), so no group waits at the merge for a second tile: 293 tokens 6.78 ->
// 6.30 us alone, forward 662.9 -> 656.9 us. Window layers from 193 to 768 tokens take 3 groups (a
// 32-query CTA reaches at most three key tiles; 192 threads, 100 KB): 293 tokens 5.92 -> 5.45 us,
// 512: 7.08 -> 6.3 us alone, forward 655.6 -> 650.0 us; at 1024 tokens the grid would take two
// waves of two CTAs an SM (10.5 against 8.2 us).
struct AttnVariant {
    int qw, ks;
    bool tc;
};
static uint32_t env_u32(const char *name, uint32_t dflt) {
    const char *e = getenv(name);
    return e ? (uint32_t)strtoul(e, nullptr, 10) : dflt;
}
// A/B knobs: the shortest global / sliding-window sequence for the tensor-core kernel.
static std::atomic<uint32_t> g_attn_tc_min{env_u32("JC_ATTN_TC_MIN", 832u)};
static std::atomic<uint32_t> g_attn_tc_min_window{env_u32("JC_ATTN_TC_MIN_WINDOW", 0xFFFFFFFFu)};
void swap_attn_tc_min(uint32_t *global_min, uint32_t *window_min) {
    *global_min = g_attn_tc_min.exchange(*global_min);
    *window_min = g_attn_tc_min_window.exchange(*window_min);
}
// Packed requests (`packed`: every row carries its request's row range) are a different regime:
// a query sees only its own request's keys, and a pack has thousands of rows. Packs of more than
// 768 rows take the tcgen05 kernel: for global layers on request-aligned tiles (the engine's
// tile list: a 128-row tile straddling two requests made the key loop pay for both), for window
// layers on plain 128-row tiles (a window bounds a tile's keys whatever it straddles). Smaller
// packs stay on the mma.sync kernel. Measured on config 3 (4096 requests): packs of up to 6144
// rows, 6428 requests/s with the tcgen05 kernel on straddling tiles for global layers, 7011 with
// 64 x 2 mma.sync CTAs for both kinds of layer (6413 with 32-query CTAs, 6928 with 32-query CTAs
// of one key group); packs of up to 12288 rows, 7551 with 64 x 2 mma.sync CTAs, 7805-7973 with
// tcgen05 window layers, 8258-8320 with request-aligned tcgen05 global layers as well
// (JC_ATTN_PACKED_GLOBAL_TC=0 keeps global layers of packs on 64 x 2 mma.sync CTAs).
static AttnVariant attn_variant(uint32_t n, uint32_t window, bool packed) {
    if (packed) {
        static const uint32_t global_tc = env_u32("JC_ATTN_PACKED_GLOBAL_TC", 1u);
        if ((window || global_tc) && n > 768) return AttnVariant{0, 0, true};
        // (the A/B knob's mma.sync shape below for global layers of big packs: 64 x 2)
    } else if (n >= (window ? g_attn_tc_min_window.load() : g_attn_tc_min.load())) {
        return AttnVariant{0, 0, true};
    }
    // A/B knob: JC_ATTN_SHAPE=<query warps><key groups>, e.g. "41".
    static const char *force = getenv("JC_ATTN_SHAPE");
    if (force && force[0] >= '1' && force[0] <= '4' && force[1] >= '1' && force[1] <= '5')
        return AttnVariant{force[0] - '0', force[1] - '0', false};
    if (packed && n > 768) return AttnVariant{4, 2, false};
    // Global attention over exactly five key tiles: one tile for each of five key groups.
    if (window == 0 && n > 256 && n <= 320) return AttnVariant{2, 5, false};
    // A 32-query CTA of a +-64 window reaches at most three key tiles: three groups of one tile,
    // while the grid (12 heads) stays within two 100 KB CTAs an SM.
    if (window > 0 && window <= 64 && n > 192 && n <= 768) return AttnVariant{2, 3, false};
    // Past 768 tokens a +-64 window's grid of 32-query CTAs takes several waves: one key group
    // a CTA (64 threads, three CTAs' worth of key tiles in flight an SM) measured best (config 4,
    // 1024 tokens: forward 925.7 us against 965.6 with two groups and 932.6 with 64-query CTAs).
    if (window > 0 && window <= 64 && n > 768) return AttnVariant{2, 1, false};
    return n > 192 && n <= 384 ? AttnVariant{2, 4, false} : AttnVariant{2, 2, false};
}

size_t attn_ws_floats(uint32_t n, uint32_t heads, uint32_t kv_chunks) {
    if (kv_chunks <= 1) return 0;
    // Enough for whichever kernel serves any length up to n.
    size_t need = 0;
    for (uint32_t qt : {32u, 64u})
        need = std::max(need, (size_t)((n + qt - 1) / qt) * heads * kv_chunks * ATTN_PART * qt * 2);
    need = std::max(need, (size_t)((n + ATC_QT - 1) / ATC_QT) * heads * kv_chunks * ATC_PART * ATC_QT);
    return need;
}

static bool launch_attn_tc(const AttnParams &p, uint32_t chunks, cudaStream_t s, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    if (!ensure_smem(attention_tc_kernel, AtcSmem::ALLOC, smem_set)) return false;
    auto fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
        return false;
    }
    AttnTcParams kp;
    kp.p = p;
    // qkv as (64 columns of a head, n rows, 3 x heads head blocks): zero fill past row n.
    cuuint64_t dims[3] = {64, p.n, 3ull * p.heads};
    cuuint64_t strides[2] = {3ull * p.heads * 64 * 2, 128};
    cuuint32_t box[3] = {64, 64, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(&kp.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(p.qkv), dims,
                    strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("attention: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
        return false;
    }
    dim3 grid(p.tiles ? attn_tile_cap(p.n) : (p.n + ATC_QT - 1) / ATC_QT, p.heads, chunks);
    return launch_ex(attention_tc_kernel, grid, dim3(ATC_THREADS), AtcSmem::ALLOC, s, pdl,
                     "attention launch", kp);
}

size_t attn_counters(uint32_t n, uint32_t heads) { return (size_t)((n + 31) / 32) * heads; }

uint32_t attention_ctas(const AttnArgs &a) {
    const AttnVariant v = attn_variant(a.n, a.window, a.seg != nullptr);
    if (v.tc && a.tiles) return attn_tile_cap(a.n) * a.heads * a.kv_chunks;
    const uint32_t qt = v.tc ? (uint32_t)ATC_QT : 16u * (uint32_t)v.qw;
    return (a.n + qt - 1) / qt * a.heads * a.kv_chunks;
}

uint32_t gemm_ctas(uint32_t m, uint32_t n, const GemmConfig &cfg) {
    const uint32_t tiles = (n / cfg.bn) * ((m + cfg.bm - 1) / cfg.bm);
    if (cfg.persistent && (cfg.bn == 128 || cfg.bn == 256) && cfg.splits == 1 && cfg.cluster == 1)
        return std::min(tiles, std::max(cfg.grid, 1u));
    return tiles * (uint32_t)(cfg.cluster > 1 ? cfg.cluster : cfg.splits);
}

// The dynamic shared memory a launch of `ctas` CTAs (each needing `need` bytes) requests so that
// an SM holds at most ceil(ctas / SMs) of them. Under programmatic dependent launch a grid's CTAs
// are placed while the previous kernel still holds most SMs: small CTAs would pack several to
// each of the few free SMs and run there in turn (a 120-CTA attention grid at 293 tokens on ~40
// SMs), instead of spreading over the SMs the previous kernel frees. One CTA more than the cap
// must not fit in an SM's shared memory (less the per-CTA reservation).
static int spread_smem(int need, uint32_t ctas) {
    static const int3 dev = []() {
        int d = 0, per_sm = 0, reserved = 0, sms = 0;
        cudaGetDevice(&d);
        cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, d);
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, d);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
        return make_int3(per_sm, reserved, sms);
    }();
    if (dev.x <= 0 || dev.z <= 0) return need;
    const uint32_t cap = (ctas + (uint32_t)dev.z - 1) / (uint32_t)dev.z;
    const int spread = ((dev.x / (int)(cap + 1) - dev.y + 1) + 127) / 128 * 128;
    return std::min(std::max(need, spread), dev.x - dev.y);
}

template <int QW, int KS>
static bool launch_attn_inst(const AttnParams &p, uint32_t chunks, cudaStream_t s, bool pdl) {
    static std::atomic<uint64_t> smem_set{0};
    using S = AttnShape<QW, KS>;
    auto kern = attention_kernel<QW, KS>;
    // Permission for any request spread_smem makes: at most a block's opt-in limit less the
    // kernel's static shared memory (the error-word slot), which the dynamic request adds to.
    static const int cap = [kern]() {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        return optin - (int)fa.sharedSizeBytes;
    }();
    if (!ensure_smem(kern, std::max(cap, S::SMEM), smem_set)) return false;
    dim3 grid((p.n + S::QT - 1) / S::QT, p.heads, chunks);
    const int smem = std::min(spread_smem(S::SMEM, grid.x * grid.y * grid.z), std::max(cap, S::SMEM));
    return launch_ex(kern, grid, dim3(S::THREADS), smem, s, pdl, "attention launch", p);
}

bool launch_attention(const AttnArgs &a, cudaStream_t s, bool pdl) {
    if (!a.qkv || !a.o || a.n == 0 || a.heads == 0) {
        set_error("attention: no input, output, rows or heads");
        return false;
    }
    if (a.kv_chunks < 1 || a.kv_chunks > 16 || (a.kv_chunks > 1 && (!a.ws || !a.counters))) {
        set_error("attention: key ranges must be 1..16, and need a workspace and counters when > 1");
        return false;
    }
    if ((reinterpret_cast<uintptr_t>(a.qkv) | reinterpret_cast<uintptr_t>(a.o)) & 15) {
        set_error("attention: qkv and o must be 16-byte aligned");
        return false;
    }
    AttnParams p{a.qkv, a.o, a.ws, a.counters, a.n, a.heads, a.window, a.seg, a.err, a.prof,
                 a.prof_cap, a.tiles};
    if (a.tiles && a.kv_chunks != 1) {
        set_error("attention: a tile list takes one key range a tile");
        return false;
    }
    const AttnVariant v = attn_variant(a.n, a.window, a.seg != nullptr);
    if (v.tc) return launch_attn_tc(p, a.kv_chunks, s, pdl);
    switch (v.qw * 10 + v.ks) {
        case 24: return launch_attn_inst<2, 4>(p, a.kv_chunks, s, pdl);
        case 42: return launch_attn_inst<4, 2>(p, a.kv_chunks, s, pdl);
        case 41: return launch_attn_inst<4, 1>(p, a.kv_chunks, s, pdl);
        case 22: return launch_attn_inst<2, 2>(p, a.kv_chunks, s, pdl);
        case 21: return launch_attn_inst<2, 1>(p, a.kv_chunks, s, pdl);
        case 25: return launch_attn_inst<2, 5>(p, a.kv_chunks, s, pdl);
        case 23: return launch_attn_inst<2, 3>(p, a.kv_chunks, s, pdl);
        default:
            set_error("attention: no compiled shape for these query warps / key groups");
            return false;
    }
}

uint32_t choose_kv_chunks(uint32_t n, uint32_t heads, uint32_t window, int sms, bool packed) {
    const AttnVariant v = attn_variant(n, window, packed);
    const uint32_t key_tiles = (n + 63) / 64;
    // Packs run the tcgen05 kernel on request-aligned tiles (one key range each).
    if (v.tc && packed) return 1;
    if (v.tc) {
        // Up to two CTAs per SM (the kernel's residency: each brings two more independent MMA
        // chains), at least two key tiles a range: the range count that minimises waves x key
        // tiles per range, ties to fewer ranges (whose merge is cheaper).
        const uint32_t tiles = ((n + ATC_QT - 1) / ATC_QT) * heads;
        const uint32_t reach = std::min(key_tiles, window ? (ATC_QT + 2 * window + 63) / 64 + 1 : key_tiles);
        uint32_t best = 1, best_cost = ~0u;
        for (uint32_t c = 1; c <= 8; c++) {
            if (c > 1 && reach < 2 * c) break;
            const uint32_t waves = (tiles * c + 2 * (uint32_t)sms - 1) / (2 * (uint32_t)sms);
            const uint32_t cost = waves * ((reach + c - 1) / c);
            if (cost < best_cost) {
                best_cost = cost;
                best = c;
            }
        }
        return best;
    }
    // Split the keys across CTAs only when a (query tile, head) grid leaves most SMs idle and each
    // key group would still walk several key tiles.
    if (window > 0) return 1;
    const uint32_t qt = 16 * v.qw;
    const uint32_t tiles = ((n + qt - 1) / qt) * heads;
    if (2 * tiles >= (uint32_t)sms || key_tiles <= (uint32_t)(2 * v.ks)) return 1;
    uint32_t c = (uint32_t)sms / (tiles ? tiles : 1);
    if (c > key_tiles / v.ks) c = key_tiles / v.ks;
    if (c > 8) c = 8;
    return c < 1 ? 1 : c;
}

// ---------------------------------------------------------------------------------------------
// edges


bool launch_embed(const uint32_t *ids, uint32_t n, const __half *table, const float *gamma,
                  uint32_t d, float eps, __half *x, float *stats, cudaStream_t s, bool pdl) {
    if (n == 0) return true;
    dim3 grid((n + 3) / 4), block(128);
#define JC_EMBED(DD) \
    case DD: return launch_ex(embed_kernel<DD>, grid, block, 0, s, pdl, "embed launch", ids, n, table, gamma, eps, x, stats);
    switch (d) {
        JC_EMBED(128) JC_EMBED(256) JC_EMBED(384) JC_EMBED(512) JC_EMBED(640) JC_EMBED(768)
        JC_EMBED(896) JC_EMBED(1024)
        default: set_error("embed: width must be a multiple of 128 up to 1024"); return false;
    }
#undef JC_EMBED
}

bool launch_norm_add(const __half *x, uint32_t n, uint32_t d, const float *gamma,
                     const float *add, float eps, __half *out, float *stats, cudaStream_t s,
                     bool pdl) {
    if (n == 0) return true;
    dim3 grid((n + 3) / 4), block(128);
#define JC_NA(DD) \
    case DD: return launch_ex(norm_add_kernel<DD>, grid, block, 0, s, pdl, "norm_add launch", x, n, gamma, add, eps, out, stats);
    switch (d) {
        JC_NA(128) JC_NA(256) JC_NA(384) JC_NA(512) JC_NA(640) JC_NA(768) JC_NA(896) JC_NA(1024)
        default: set_error("norm_add: width must be a multiple of 128 up to 1024"); return false;
    }
#undef JC_NA
}

bool launch_gather_rows(const __half *x, const float *stats, uint32_t d, const uint32_t *rows,
                        uint32_t k, uint32_t limit, __half *out, float *out_stats, cudaStream_t s,
                        bool pdl, unsigned int *err) {
    if (k == 0) return true;
    if (d % 8) {
        set_error("gather: width must be a multiple of 8");
        return false;
    }
    return launch_ex(gather_rows_kernel, dim3((k + 3) / 4), dim3(128), 0, s, pdl, "gather launch",
                     x, stats, d, rows, k, limit, out, out_stats, err);
}

bool launch_score(const __half *y, uint32_t d, const __half *w, float b, const uint32_t *markers,
                  uint32_t k, float *logits, cudaStream_t s, bool pdl) {
    if (k == 0) return true;
    if (d % 2) {
        set_error("score: width must be even");
        return false;
    }
    return launch_ex(score_kernel, dim3((k + 3) / 4), dim3(128), 0, s, pdl, "score launch", y, d,
                     w, b, markers, k, logits);
}

// ---------------------------------------------------------------------------------------------
// persistent kernel

int persist_blocks_per_sm() {
    static std::atomic<uint64_t> smem_set{0};
    if (!ensure_smem(persist_kernel, PERSIST_SMEM, smem_set)) return 0;
    int per_sm = 0;
    if (!cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, persist_kernel,
                                                               PERSIST_THREADS, PERSIST_SMEM),
                 "occupancy"))
        return 0;
    return per_sm;
}

// The in-forward time (us) of one 128-row GEMM tile of width bn over depth k, as the phase stamps
// of the per-step kernels measure it on a B200 (profiles/forward_293_phase_stamps.md): first
// stage and drain 0.8 us, the main loop 0.163 us per 64-deep k-block whatever the tile's width
// (or height, or number of MMA issuer warps), the epilogue 0.70 us per 32 columns a
// row holds. The B200 restatement of the reference's per-task cost (src/forward.rs:783-806:
// 5 us a task plus 0.35 us a K step on 68 SMs).
double gemm_tile_us(uint32_t k, int bn) {
    return 0.8 + 0.163 * (double)((k + GEMM_BK - 1) / GEMM_BK) + 0.70 * (double)bn / 32.0;
}

// A phase's time on `grid` CTAs: its tiles in waves.
double gemm_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid) {
    const uint64_t tiles = (uint64_t)((m + GEMM_BM - 1) / GEMM_BM) * (n / (uint32_t)bn);
    const uint64_t waves = (tiles + grid - 1) / std::max(grid, 1u);
    return (double)waves * gemm_tile_us(k, bn);
}

// A phase of the persistent kernel: phase_us plus what its items cost a row block's completion.
// Every item of a row block reports to the block's counter and the next phase's items of that
// block wait for all of them: each item adds about 0.19 us (fitted to the whole-model forward at
// 293 tokens: 32-column phases for the 768-wide GEMMs measured 1067.8 against 991.7 us with
// 64-column ones, +1.55 us a phase where the tile time alone predicts -0.70 us, for 12 more items
// a row block).
double persist_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid) {
    return gemm_phase_us(m, n, k, bn, grid) + 0.19 * (double)(n / (uint32_t)bn);
}

// Tile width policy of the persistent kernel: 0 (the plan), 64 or 32 (every phase that allows
// it); a tuning and test hook (jc_persist_tile_policy), JC_PERSIST_BN sets its start value.
static std::atomic<int> g_persist_bn{(int)env_u32_early("JC_PERSIST_BN", 0u)};
void swap_persist_tile_policy(int *bn) { *bn = g_persist_bn.exchange(*bn); }

// The persistent kernel's tile width for a GEMM phase (the B200 counterpart of the reference's
// gemm_plan, src/forward.rs:761-769): 64 or 32 columns, whichever persist_phase_us finds cheaper
// on the launch's grid (ties to 64); RoPE and GeGLU keep 64 (their column pairs span a 64-wide
// chunk).
uint32_t persist_tile_width(uint32_t m, uint32_t n, uint32_t k, uint32_t epi, uint32_t grid) {
    if ((epi & (JC_EPI_ROPE | JC_EPI_GEGLU)) || n % PERSIST_BN_NARROW) return PERSIST_BN;
    if (n % PERSIST_BN) return PERSIST_BN_NARROW;
    const int policy = g_persist_bn.load();
    if (policy == PERSIST_BN || policy == PERSIST_BN_NARROW) return (uint32_t)policy;
    return persist_phase_us(m, n, k, PERSIST_BN_NARROW, grid) < persist_phase_us(m, n, k, PERSIST_BN, grid)
               ? PERSIST_BN_NARROW
               : PERSIST_BN;
}

uint32_t plan_flow(PhaseDesc *d, uint32_t n, uint32_t grid) {
    uint32_t first = 0;
    for (uint32_t i = 0; i < n; i++) {
        PhaseDesc &p = d[i];
        p.bn = 0;
        if (p.kind == PH_GEMM) {
            p.rows = p.g.m;
            p.bn = persist_tile_width(p.g.m, p.g.n, p.g.k, p.epi, grid);
            p.items = (p.g.m + GEMM_BM - 1) / GEMM_BM * (p.g.n / p.bn);
        } else if (p.kind == PH_ATTN) {
            p.rows = p.a.n;
            p.items = (p.a.n + FLOW_CHUNK - 1) / FLOW_CHUNK * p.a.heads;
        } else {
            p.rows = p.r.n;
            p.items = (p.r.n + FLOW_ROWS - 1) / FLOW_ROWS;
        }
        p.first_item = first;
        first += p.items;
        p.extra = 0;
        p.dep[0] = PhaseDep{DEP_NONE, 0, 0};
        p.dep[1] = PhaseDep{DEP_NONE, 0, 0};
        if (i > 0) {
            // The previous phase's output is this phase's input: the same rows, except attention
            // (keys within the window, or every key) and the marker gather (any row).
            if (p.kind == PH_ATTN)
                p.dep[0] = p.a.window ? PhaseDep{DEP_WINDOW, i - 1, p.a.window} : PhaseDep{DEP_ALL, i - 1, 0};
            else
                p.dep[0] = PhaseDep{p.kind == PH_GATHER ? DEP_ALL : DEP_ROWS, i - 1, 0};
        }
        // A GEMM that overwrites an attention phase's qkv input also waits for every task that
        // may still read the rows it writes (write after read).
        if (p.kind == PH_GEMM)
            for (uint32_t j = i; j-- > 0;)
                if (d[j].kind == PH_ATTN && d[j].a.qkv == p.g.c) {
                    p.dep[1] = d[j].a.window ? PhaseDep{DEP_WINDOW, j, d[j].a.window} : PhaseDep{DEP_ALL, j, 0};
                    break;
                }
    }
    return first;
}

bool launch_persist(const PhaseDesc *phases, uint32_t n_phases, uint32_t total_items, uint32_t *ctr,
                    uint32_t blocks, uint32_t grid, uint64_t timeout_ns, cudaStream_t s,
                    unsigned int *err, uint64_t *prof, uint32_t prof_cap) {
    static std::atomic<uint64_t> smem_set{0};
    if (!ensure_smem(persist_kernel, PERSIST_SMEM, smem_set)) return false;
    FlowParams P{phases, n_phases, total_items, blocks, ctr, timeout_ns, err, prof, prof ? prof_cap : 0u};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(PERSIST_THREADS);
    cfg.dynamicSmemBytes = PERSIST_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_ok(cudaLaunchKernelEx(&cfg, persist_kernel, P), "persistent kernel launch");
}

}  // namespace jc
