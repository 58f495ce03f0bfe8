// The C ABI (include/julia_cuda.h): the reference's julia_cuda_* entry points (src/capi.rs), the
// added raw-model / device-pointer entry points, the per-kernel entry points and host prep.
// Every entry point catches C++ exceptions and reports them as errors.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <fstream>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/julia_cuda.h"
#include "checkpoint.h"
#include "engine.h"
#include "jc_internal.h"
#include "model.h"

struct JcEngine {
    jc::Engine *e;
};

namespace {

void report(char *err, size_t len, const std::string &msg) {
    jc::set_error(msg);
    if (!err || len == 0) return;
    const size_t n = std::min(msg.size(), len - 1);
    std::memcpy(err, msg.data(), n);
    err[n] = 0;
}

template <typename F>
auto guarded(char *err, size_t len, F &&f) -> decltype(f()) {
    try {
        return f();
    } catch (const std::exception &ex) {
        report(err, len, std::string("julia-cuda: exception: ") + ex.what());
    } catch (...) {
        report(err, len, "julia-cuda: unknown exception");
    }
    // Failure: -1 for the int-returning entry points, NULL for the pointer-returning ones.
    if constexpr (std::is_same_v<decltype(f()), int>)
        return -1;
    else
        return decltype(f())();
}

bool set_device(int dev, char *err, size_t len) {
    cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) {
        report(err, len, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
        return false;
    }
    return true;
}

}  // namespace

extern "C" {

const char *julia_cuda_tier(void) { return "sm_100a"; }

void julia_cuda_default_config(jc_model_config *c) {
    c->d_model = 768;
    c->n_heads = 12;
    c->inter = 1152;
    c->n_layers = 22;
    c->vocab = 50368;
    c->head_ff = 2048;
    c->scorer_hidden = 384;
    c->n_head_layers = 2;
    c->global_every = 3;
    c->window = 64;
    c->max_positions = 8192;
    c->n_qtypes = 3;
    c->norm_eps = 1e-5f;
    c->head_eps = 1e-5f;
    c->theta_global = 160000.0f;
    c->theta_local = 10000.0f;
}

size_t julia_cuda_raw_size(const jc_model_config *cfg) {
    std::string why;
    if (!cfg || !jc::check_config(*cfg, &why)) return 0;
    return jc::raw_layout(*cfg).total;
}

int julia_cuda_raw_offsets(const jc_model_config *cfg, size_t *offsets, size_t cap) {
    std::string why;
    if (!cfg || !jc::check_config(*cfg, &why)) {
        jc::set_error(why);
        return -1;
    }
    const jc::RawLayout L = jc::raw_layout(*cfg);
    for (size_t i = 0; i < L.order.size() && i < cap; i++) offsets[i] = L.order[i].off;
    return (int)L.order.size();
}

void julia_cuda_init_random(const jc_model_config *cfg, uint64_t seed, float *raw) {
    std::string why;
    if (!cfg || !raw || !jc::check_config(*cfg, &why)) return;
    jc::init_random(*cfg, seed, raw);
}

int julia_cuda_save_raw(const char *dir, const jc_model_config *cfg, const float *raw, char *err,
                        size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        std::string why;
        if (!dir || !cfg || !raw || !jc::check_config(*cfg, &why)) {
            report(err, err_len, "save: " + (why.empty() ? std::string("null argument") : why));
            return -1;
        }
        const size_t n = jc::raw_layout(*cfg).total;
        std::ofstream c(std::string(dir) + "/jc_config.bin", std::ios::binary);
        c.write(reinterpret_cast<const char *>(cfg), sizeof(*cfg));
        std::ofstream w(std::string(dir) + "/jc_weights.f32", std::ios::binary);
        w.write(reinterpret_cast<const char *>(raw), (std::streamsize)(n * 4));
        if (!c || !w) {
            report(err, err_len, std::string("save: cannot write to ") + dir);
            return -1;
        }
        return 0;
    });
}

int julia_cuda_read_checkpoint(const char *dir, jc_model_config *cfg, float *raw, size_t raw_cap,
                               size_t *raw_len, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!dir || !cfg) {
            report(err, err_len, "read_checkpoint: null directory or config");
            return -1;
        }
        std::vector<float> r;
        std::string why;
        if (!jc::read_checkpoint(dir, cfg, &r, &why)) {
            report(err, err_len, "read_checkpoint: " + why);
            return -1;
        }
        if (raw_len) *raw_len = r.size();
        if (raw) {
            if (raw_cap < r.size()) {
                report(err, err_len, "read_checkpoint: raw holds " + std::to_string(raw_cap) +
                                         " floats, the model needs " + std::to_string(r.size()));
                return -1;
            }
            std::memcpy(raw, r.data(), r.size() * 4);
        }
        return 0;
    });
}

int julia_cuda_save_checkpoint(const char *dir, const jc_model_config *cfg, const float *raw,
                               int dtype, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        std::string why;
        if (!dir || !cfg || !raw) {
            report(err, err_len, "save_checkpoint: null argument");
            return -1;
        }
        if (!jc::write_checkpoint(dir, *cfg, raw, dtype, &why)) {
            report(err, err_len, "save_checkpoint: " + why);
            return -1;
        }
        return 0;
    });
}

int julia_cuda_prepare_host(const jc_model_config *cfg, const float *raw, size_t raw_len,
                            size_t max_length, uint16_t *f16, size_t f16_cap, float *f32,
                            size_t f32_cap, size_t *f16_len, size_t *f32_len, char *err,
                            size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        std::string why;
        if (!cfg || !raw || !jc::check_config(*cfg, &why) || raw_len != jc::raw_layout(*cfg).total) {
            report(err, err_len, "prepare: " + (why.empty() ? std::string("bad arguments") : why));
            return -1;
        }
        const size_t L = max_length ? max_length : (size_t)cfg->max_positions;
        jc::HostWeights hw;
        if (!jc::prepare_weights(*cfg, raw, (uint32_t)L, &hw, &why)) {
            report(err, err_len, "prepare: " + why);
            return -1;
        }
        if (f16_len) *f16_len = hw.f16.size();
        if (f32_len) *f32_len = hw.f32.size();
        if ((f16 && f16_cap < hw.f16.size()) || (f32 && f32_cap < hw.f32.size())) {
            report(err, err_len, "prepare: the output arrays are too small");
            return -1;
        }
        if (f16) std::memcpy(f16, hw.f16.data(), hw.f16.size() * 2);
        if (f32) std::memcpy(f32, hw.f32.data(), hw.f32.size() * 4);
        return 0;
    });
}

JcEngine *julia_cuda_load_raw(const jc_model_config *cfg, const float *raw, size_t raw_len,
                              size_t max_length, int device, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> JcEngine * {
        std::string why;
        if (!cfg || !raw) {
            report(err, err_len, "load: null config or weights");
            return nullptr;
        }
        if (!jc::check_config(*cfg, &why)) {
            report(err, err_len, "load: " + why);
            return nullptr;
        }
        if (raw_len != jc::raw_layout(*cfg).total) {
            report(err, err_len, "load: the weights are not the size the config describes");
            return nullptr;
        }
        jc::Engine *e = jc::Engine::create(*cfg, raw, max_length, device, &why);
        if (!e) {
            report(err, err_len, "load: " + why);
            return nullptr;
        }
        return new JcEngine{e};
    });
}

JcEngine *julia_cuda_load_random(const jc_model_config *cfg, uint64_t seed, size_t max_length,
                                 int device, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> JcEngine * {
        std::string why;
        if (!cfg || !jc::check_config(*cfg, &why)) {
            report(err, err_len, "load: " + (why.empty() ? std::string("null config") : why));
            return nullptr;
        }
        std::vector<float> raw(jc::raw_layout(*cfg).total);
        jc::init_random(*cfg, seed, raw.data());
        return julia_cuda_load_raw(cfg, raw.data(), raw.size(), max_length, device, err, err_len);
    });
}

JcEngine *julia_cuda_load(const char *dir, size_t max_length, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> JcEngine * {
        if (!dir) {
            report(err, err_len, "load: null directory");
            return nullptr;
        }
        if (jc::has_checkpoint(dir)) {
            // The reference's checkpoint layout: model.safetensors + encoder/config.json +
            // julia_config.json (src/checkpoint.rs:27-62).
            jc_model_config cfg;
            std::vector<float> raw;
            std::string why;
            if (!jc::read_checkpoint(dir, &cfg, &raw, &why)) {
                report(err, err_len, "load: " + why);
                return nullptr;
            }
            return julia_cuda_load_raw(&cfg, raw.data(), raw.size(), max_length, 0, err, err_len);
        }
        jc_model_config cfg;
        std::ifstream c(std::string(dir) + "/jc_config.bin", std::ios::binary);
        if (!c.read(reinterpret_cast<char *>(&cfg), sizeof(cfg))) {
            report(err, err_len, std::string("load: no model at ") + dir +
                                     " (model.safetensors + encoder/config.json + "
                                     "julia_config.json, or jc_config.bin + jc_weights.f32)");
            return nullptr;
        }
        std::string why;
        if (!jc::check_config(cfg, &why)) {
            report(err, err_len, "load: " + why);
            return nullptr;
        }
        const size_t n = jc::raw_layout(cfg).total;
        std::vector<float> raw(n);
        std::ifstream w(std::string(dir) + "/jc_weights.f32", std::ios::binary);
        if (!w.read(reinterpret_cast<char *>(raw.data()), (std::streamsize)(n * 4))) {
            report(err, err_len, std::string("load: jc_weights.f32 in ") + dir + " is short");
            return nullptr;
        }
        return julia_cuda_load_raw(&cfg, raw.data(), n, max_length, 0, err, err_len);
    });
}

void julia_cuda_free(JcEngine *engine) {
    if (!engine) return;
    try {
        delete engine->e;
    } catch (...) {
    }
    delete engine;
}

void julia_cuda_device(const JcEngine *engine, char *buf, size_t len) {
    if (!engine) return;
    report(buf, len, engine->e->name);
}

int julia_cuda_engine_config(const JcEngine *engine, jc_model_config *cfg, size_t *max_length,
                             int *device, int *sms) {
    if (!engine) return -1;
    if (cfg) *cfg = engine->e->cfg;
    if (max_length) *max_length = engine->e->max_length;
    if (device) *device = engine->e->device;
    if (sms) *sms = engine->e->sms;
    return 0;
}

int julia_cuda_set_packing(JcEngine *engine, size_t rows) {
    if (!engine || rows > engine->e->max_length) return -1;
    engine->e->pack_rows = rows;
    return 0;
}

int julia_cuda_set_head_length(JcEngine *engine, size_t rows) {
    if (!engine) return -1;
    engine->e->head_length = rows;
    return 0;
}

int julia_cuda_launches_per_forward(const JcEngine *engine, uint32_t n, uint32_t n_markers,
                                    int layer_fused) {
    if (!engine) return -1;
    return engine->e->launches_per_forward(n, n_markers, layer_fused);
}

int julia_cuda_barrier_timeout_probe(JcEngine *engine, uint64_t timeout_ns, uint32_t *code,
                                     char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!engine || !code) {
            report(err, err_len, "probe: null engine or code");
            return -1;
        }
        if (!set_device(engine->e->device, err, err_len)) return -1;
        if (!engine->e->barrier_timeout_probe(timeout_ns, code)) {
            report(err, err_len, std::string("probe: ") + jc::last_error());
            return -1;
        }
        return 0;
    });
}

int julia_cuda_device_error(JcEngine *engine, uint32_t *code, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!engine || !code) {
            report(err, err_len, "device_error: null engine or code");
            return -1;
        }
        if (!set_device(engine->e->device, err, err_len)) return -1;
        unsigned int c = 0;
        if (!engine->e->take_device_error(&c)) {
            report(err, err_len, std::string("device_error: ") + jc::last_error());
            return -1;
        }
        *code = c;
        return 0;
    });
}

}  // extern "C"

// The device-pointer forward, optionally traced (julia_cuda_forward_device / _trace).
static int forward_on_device(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                             const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                             int layer_fused, float *d_logits, const jc::Trace &tr, void *stream,
                             char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!engine) {
            report(err, err_len, "forward: null engine");
            return -1;
        }
        jc::Engine *e = engine->e;
        if (!set_device(e->device, err, err_len)) return -1;
        if (n == 0 || n > e->max_length || n_markers > e->max_length) {
            report(err, err_len, "forward: " + std::to_string(n) + " tokens / " +
                                     std::to_string(n_markers) + " markers, limit " +
                                     std::to_string(e->max_length));
            return -1;
        }
        cudaStream_t s = (cudaStream_t)stream;
        if (!jc::cuda_ok(cudaMemcpyAsync(e->ids, d_ids, n * 4, cudaMemcpyDeviceToDevice, s), "ids") ||
            (n_markers && !jc::cuda_ok(cudaMemcpyAsync(e->markers, d_markers, n_markers * 4,
                                                       cudaMemcpyDeviceToDevice, s),
                                       "markers"))) {
            report(err, err_len, jc::last_error());
            return -1;
        }
        const bool traced = tr.enc || tr.head || tr.scorer;
        const bool ok = traced ? e->enqueue_forward(n, n_markers, qtype, layer_fused, tr, s)
                               : e->launch_forward(n, n_markers, qtype, layer_fused, s);
        if (!ok) {
            report(err, err_len, std::string("forward: ") + jc::last_error());
            return -1;
        }
        if (n_markers && !jc::cuda_ok(cudaMemcpyAsync(d_logits, e->logits, n_markers * 4,
                                                      cudaMemcpyDeviceToDevice, s),
                                      "logits")) {
            report(err, err_len, jc::last_error());
            return -1;
        }
        return 0;
    });
}

extern "C" {

int julia_cuda_forward_device(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                              const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                              int layer_fused, float *d_logits, uint16_t *d_trace, void *stream,
                              char *err, size_t err_len) {
    jc::Trace tr;
    tr.enc = d_trace;
    return forward_on_device(engine, d_ids, n, d_markers, n_markers, qtype, layer_fused, d_logits,
                             tr, stream, err, err_len);
}

int julia_cuda_forward_trace(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                             const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                             int layer_fused, float *d_logits, uint16_t *d_trace,
                             uint16_t *d_head_trace, uint16_t *d_scorer_trace, void *stream,
                             char *err, size_t err_len) {
    jc::Trace tr;
    tr.enc = d_trace;
    tr.head = d_head_trace;
    tr.scorer = d_scorer_trace;
    return forward_on_device(engine, d_ids, n, d_markers, n_markers, qtype, layer_fused, d_logits,
                             tr, stream, err, err_len);
}

int julia_cuda_forward_profile(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                               const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                               float *d_logits, uint64_t *d_prof, uint32_t records_per_launch,
                               jc_launch_info *info, size_t info_cap, size_t *n_launches,
                               void *stream, char *err, size_t err_len) {
    return julia_cuda_forward_profile_mode(engine, d_ids, n, d_markers, n_markers, qtype, 0,
                                           d_logits, d_prof, records_per_launch, info, info_cap,
                                           n_launches, stream, err, err_len);
}

int julia_cuda_forward_profile_mode(JcEngine *engine, const uint32_t *d_ids, uint32_t n,
                                    const uint32_t *d_markers, uint32_t n_markers, uint32_t qtype,
                                    int layer_fused, float *d_logits, uint64_t *d_prof,
                                    uint32_t records_per_launch, jc_launch_info *info,
                                    size_t info_cap, size_t *n_launches, void *stream, char *err,
                                    size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!engine || !d_prof || records_per_launch == 0) {
            report(err, err_len, "profile: null engine or record array");
            return -1;
        }
        if (layer_fused < jc::MODE_STEPS || layer_fused > jc::MODE_MODEL) {
            report(err, err_len, "profile: no execution mode " + std::to_string(layer_fused));
            return -1;
        }
        jc::Engine *e = engine->e;
        if (!set_device(e->device, err, err_len)) return -1;
        if (n == 0 || n > e->max_length || n_markers > e->max_length) {
            report(err, err_len, "profile: " + std::to_string(n) + " tokens / " +
                                     std::to_string(n_markers) + " markers, limit " +
                                     std::to_string(e->max_length));
            return -1;
        }
        cudaStream_t s = (cudaStream_t)stream;
        if (!jc::cuda_ok(cudaMemcpyAsync(e->ids, d_ids, n * 4, cudaMemcpyDeviceToDevice, s), "ids") ||
            (n_markers && !jc::cuda_ok(cudaMemcpyAsync(e->markers, d_markers, n_markers * 4,
                                                       cudaMemcpyDeviceToDevice, s),
                                       "markers"))) {
            report(err, err_len, jc::last_error());
            return -1;
        }
        std::vector<jc_launch_info> log;
        jc::Trace tr;
        tr.prof = d_prof;
        tr.prof_cap = records_per_launch;
        if (layer_fused != jc::MODE_STEPS) {
            // Persistent modes run on `stream` directly (their phase list is uploaded per call).
            e->launch_log = &log;
            const bool ok = e->enqueue_forward(n, n_markers, qtype, layer_fused, tr, s);
            e->launch_log = nullptr;
            if (!ok || (n_markers && !jc::cuda_ok(cudaMemcpyAsync(d_logits, e->logits, n_markers * 4,
                                                                  cudaMemcpyDeviceToDevice, s),
                                                  "logits")) ||
                !jc::cuda_ok(cudaStreamSynchronize(s), "profile")) {
                report(err, err_len, std::string("profile: ") + jc::last_error());
                return -1;
            }
            if (n_launches) *n_launches = log.size();
            for (size_t i = 0; info && i < log.size() && i < info_cap; i++) info[i] = log[i];
            return 0;
        }
        // The forward captured into a CUDA graph (with its programmatic dependent launches) on
        // the engine's stream, as julia_cuda_run's forwards are, then run on `stream`.
        cudaStream_t cap = e->stream;
        if (!jc::cuda_ok(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "begin capture")) {
            report(err, err_len, std::string("profile: ") + jc::last_error());
            return -1;
        }
        e->launch_log = &log;
        const bool ok = e->enqueue_forward(n, n_markers, qtype, jc::MODE_STEPS, tr, cap);
        e->launch_log = nullptr;
        cudaGraph_t graph = nullptr;
        cudaError_t ce = cudaStreamEndCapture(cap, &graph);
        if (!ok || !jc::cuda_ok(ce, "end capture")) {
            if (graph) cudaGraphDestroy(graph);
            report(err, err_len, std::string("profile: ") + jc::last_error());
            return -1;
        }
        cudaGraphExec_t exec = nullptr;
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (!jc::cuda_ok(ce, "graph instantiate")) {
            report(err, err_len, std::string("profile: ") + jc::last_error());
            return -1;
        }
        const bool ran = jc::cuda_ok(cudaGraphLaunch(exec, s), "graph launch") &&
                         (n_markers == 0 ||
                          jc::cuda_ok(cudaMemcpyAsync(d_logits, e->logits, n_markers * 4,
                                                      cudaMemcpyDeviceToDevice, s),
                                      "logits")) &&
                         jc::cuda_ok(cudaStreamSynchronize(s), "profile");
        cudaGraphExecDestroy(exec);
        if (!ran) {
            report(err, err_len, std::string("profile: ") + jc::last_error());
            return -1;
        }
        if (n_launches) *n_launches = log.size();
        for (size_t i = 0; info && i < log.size() && i < info_cap; i++) info[i] = log[i];
        return 0;
    });
}

int julia_cuda_run(const JcEngine *engine, size_t b, const uint32_t *ids, const size_t *lens,
                   const uint32_t *markers, const size_t *n_markers, const uint32_t *qtypes,
                   int layer_fused, float *logits, float *gpu_ms, char *err, size_t err_len) {
    return guarded(err, err_len, [&]() -> int {
        if (!engine) {
            report(err, err_len, "run: null engine");
            return -1;
        }
        jc::Engine *e = engine->e;
        if (!set_device(e->device, err, err_len)) return -1;
        // Validate every sequence before queueing any (src/capi.rs:154-179).
        size_t at_id = 0, at_mk = 0;
        for (size_t i = 0; i < b; i++) {
            if (qtypes[i] >= (uint32_t)e->cfg.n_qtypes) {
                report(err, err_len, "sequence " + std::to_string(i) + ": no question type " +
                                         std::to_string(qtypes[i]));
                return -1;
            }
            if (lens[i] == 0 || lens[i] > e->max_length) {
                report(err, err_len, "sequence " + std::to_string(i) + ": " + std::to_string(lens[i]) +
                                         " tokens, not 1 to " + std::to_string(e->max_length));
                return -1;
            }
            if (n_markers[i] > e->max_length) {
                report(err, err_len, "sequence " + std::to_string(i) + ": too many markers");
                return -1;
            }
            for (size_t j = 0; j < lens[i]; j++)
                if (ids[at_id + j] >= (uint32_t)e->cfg.vocab) {
                    report(err, err_len, "sequence " + std::to_string(i) + ": token id " +
                                             std::to_string(ids[at_id + j]) + " is past the vocabulary");
                    return -1;
                }
            const size_t head = e->head_rows((uint32_t)lens[i]);
            for (size_t j = 0; j < n_markers[i]; j++)
                if (markers[at_mk + j] >= head) {
                    report(err, err_len, "sequence " + std::to_string(i) + ": a marker is past the " +
                                             (head < lens[i] ? "head's rows" : "sequence"));
                    return -1;
                }
            at_id += lens[i];
            at_mk += n_markers[i];
        }
        const size_t L = e->max_length;
        cudaStream_t s = e->stream;
        // Forwards: each request alone, or (packing on, no head length) consecutive requests of
        // one question type packed while their rows fit pack_rows and their markers L.
        struct Forward {
            size_t first, last, rows, marks, id0, mk0;
        };
        std::vector<Forward> fwd;
        const bool pack = e->pack_rows > 0 && e->head_length == 0;
        at_id = at_mk = 0;
        for (size_t i = 0; i < b; i++) {
            Forward *f = fwd.empty() ? nullptr : &fwd.back();
            if (pack && f && qtypes[f->first] == qtypes[i] && f->rows + lens[i] <= e->pack_rows &&
                f->marks + n_markers[i] <= L) {
                f->last = i + 1;
                f->rows += lens[i];
                f->marks += n_markers[i];
            } else {
                fwd.push_back(Forward{i, i + 1, lens[i], n_markers[i], at_id, at_mk});
            }
            at_id += lens[i];
            at_mk += n_markers[i];
        }
        size_t out_at = 0;
        for (size_t c0 = 0; c0 < fwd.size(); c0 += jc::Engine::QUEUE) {
            const size_t c1 = std::min(fwd.size(), c0 + (size_t)jc::Engine::QUEUE);
            for (size_t fi = c0; fi < c1; fi++) {
                const Forward &f = fwd[fi];
                const int slot = (int)(fi - c0);
                const bool packed = f.last - f.first > 1;
                // ids at [0, rows), markers at [L, L + marks) (rows of the packed forward), and
                // for packed forwards each row's request rows at [2L, 2L + 2 rows): as on the
                // device, so the forward's inputs are one copy.
                // Packed forwards are padded to 64-row / 8-marker buckets (padding rows form a
                // segment of their own, padding markers read row 0 and are dropped), so a few
                // CUDA graphs serve every pack.
                const size_t rows = packed ? std::min(L, (f.rows + 63) / 64 * 64) : f.rows;
                const size_t marks = packed ? std::min(L, (f.marks + 7) / 8 * 8) : f.marks;
                uint32_t *stage = e->h_ids + slot * e->input_words();
                std::memcpy(stage, ids + f.id0, f.rows * 4);
                uint32_t row = 0, mk = 0;
                size_t m_src = f.mk0;  // request i's markers: markers[m_src, m_src + n_markers[i])
                for (size_t i = f.first; i < f.last; i++) {
                    const uint32_t n = (uint32_t)lens[i];
                    for (size_t j = 0; j < n_markers[i]; j++) stage[L + mk++] = row + markers[m_src + j];
                    m_src += n_markers[i];
                    if (packed)
                        for (uint32_t r = 0; r < n; r++) {
                            stage[2 * L + 2 * (row + r)] = row;
                            stage[2 * L + 2 * (row + r) + 1] = row + n;
                        }
                    row += n;
                }
                for (size_t r = f.rows; r < rows; r++) {
                    stage[r] = 0;
                    stage[2 * L + 2 * r] = (uint32_t)f.rows;
                    stage[2 * L + 2 * r + 1] = (uint32_t)rows;
                }
                for (size_t j = f.marks; j < marks; j++) stage[L + j] = 0;
                if (packed) {
                    // The tcgen05 attention's tiles: up to 128 rows of one request each (the
                    // padding rows are a request of their own), or, if they do not fit the
                    // list, the plain 128-row tiles; empty entries after them.
                    uint32_t *tl = stage + 4 * L;
                    const uint32_t cap = jc::attn_tile_cap((uint32_t)rows);
                    uint32_t t = 0;
                    bool fits = true;
                    auto add = [&](uint32_t s0, uint32_t s1) {
                        for (uint32_t q = s0; fits && q < s1; q += 128) {
                            if (t == cap) {
                                fits = false;
                                break;
                            }
                            tl[2 * t] = q;
                            tl[2 * t + 1] = std::min(q + 128, s1);
                            t++;
                        }
                    };
                    uint32_t r0 = 0;
                    for (size_t i = f.first; i < f.last; i++) {
                        add(r0, r0 + (uint32_t)lens[i]);
                        r0 += (uint32_t)lens[i];
                    }
                    add((uint32_t)f.rows, (uint32_t)rows);
                    if (!fits) {
                        t = 0;
                        for (uint32_t q = 0; q < rows; q += 128, t++) {
                            tl[2 * t] = q;
                            tl[2 * t + 1] = std::min(q + 128, (uint32_t)rows);
                        }
                    }
                    for (; t < cap; t++) tl[2 * t] = tl[2 * t + 1] = 0;
                }
                const size_t words = packed ? 4 * L + 2 * (size_t)jc::attn_tile_cap((uint32_t)rows)
                                            : (f.marks ? L + f.marks : f.rows);
                bool ok = jc::cuda_ok(cudaMemcpyAsync(e->ids, stage, words * 4, cudaMemcpyHostToDevice,
                                                      s), "ids and markers") &&
                          jc::cuda_ok(cudaEventRecord(e->ev_start[slot], s), "event") &&
                          e->launch_forward((uint32_t)rows, (uint32_t)marks, qtypes[f.first],
                                            layer_fused, s, packed) &&
                          jc::cuda_ok(cudaEventRecord(e->ev_end[slot], s), "event") &&
                          (f.marks == 0 || jc::cuda_ok(cudaMemcpyAsync(e->h_logits + slot * L, e->logits,
                                                                       f.marks * 4, cudaMemcpyDeviceToHost, s),
                                                       "logits"));
                if (!ok) {
                    cudaStreamSynchronize(s);
                    report(err, err_len, std::string("run: ") + jc::last_error());
                    return -1;
                }
            }
            if (!jc::enqueue_device_error_read(e->h_err, s, e->dev_err) ||
                !jc::cuda_ok(cudaStreamSynchronize(s), "run")) {
                report(err, err_len, std::string("run: ") + jc::last_error());
                return -1;
            }
            std::string why;
            if (!e->check_device_error_copy(&why)) {
                report(err, err_len, "run: " + why);
                return -1;
            }
            for (size_t fi = c0; fi < c1; fi++) {
                const Forward &f = fwd[fi];
                const int slot = (int)(fi - c0);
                for (size_t j = 0; j < f.marks; j++) {
                    const float v = e->h_logits[slot * L + j];
                    if (!std::isfinite(v)) {
                        report(err, err_len, "run: inference returned nonfinite logits");
                        return -1;
                    }
                    logits[out_at + j] = v;
                }
                out_at += f.marks;
                float ms = 0.f;
                cudaEventElapsedTime(&ms, e->ev_start[slot], e->ev_end[slot]);
                for (size_t i = f.first; i < f.last; i++) gpu_ms[i] = ms;  // a packed forward's time
            }
        }
        return 0;
    });
}

// ------------------------------------------------------------------------------------------
// per-kernel entry points

const char *jc_last_error(void) { return jc::last_error(); }

int jc_device_error(uint32_t *code) {
    unsigned int c = 0;
    if (!jc::read_device_error(&c, nullptr)) return -1;
    if (code) *code = c;
    return 0;
}

static jc::GemmConfig pick(uint32_t m, uint32_t n, uint32_t k, int bn, int splits, uint32_t epi) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    jc::GemmConfig c = jc::choose_gemm(m, n, k, sms);
    if ((epi & (JC_EPI_ROPE | JC_EPI_GEGLU)) && c.bn < 64) c.bn = 64;
    if (bn) c.bn = bn;
    jc::request_splits(c, splits);
    jc::set_gemm_depth(c, m, n, sms);
    return c;
}

size_t jc_gemm_ws_floats(uint32_t m, uint32_t n, uint32_t k, int bn, int splits) {
    return jc::gemm_ws_floats(m, n, pick(m, n, k, bn, splits, 0));
}

size_t jc_gemm_counters(uint32_t m, uint32_t n, uint32_t k, int bn, int splits) {
    return jc::gemm_counters(m, n, pick(m, n, k, bn, splits, 0));
}

int jc_choose_gemm(uint32_t m, uint32_t n, uint32_t k, int sms, int *bn, int *splits) {
    jc::GemmConfig c = jc::choose_gemm(m, n, k, sms);
    if (bn) *bn = c.bn;
    if (splits) *splits = c.cluster > 1 ? -c.cluster : c.splits;
    return 0;
}

int jc_gemm(uint32_t epi, int bn, int splits, const uint16_t *a, const uint16_t *w, uint16_t *c,
            const uint16_t *res, float *ws, uint32_t *counters, const float *stats_in,
            const float *colsum, float *stats_out, float *zero, uint32_t zero_len, uint32_t m,
            uint32_t n, uint32_t k, float eps, const float *rope, const float *bias, void *stream) {
    return guarded(nullptr, 0, [&]() -> int {
        if (!a || !w) {
            jc::set_error("gemm: null a or w");
            return -1;
        }
        jc::GemmConfig cfg = pick(m, n, k, bn, splits, epi);
        jc::GemmArgs g;
        g.epi = epi;
        g.c = reinterpret_cast<__half *>(c);
        g.res = reinterpret_cast<const __half *>(res);
        g.ws = ws;
        g.counters = counters;
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
        return jc::launch_gemm(g, cfg, (cudaStream_t)stream, true) ? 0 : -1;
    });
}

size_t jc_attention_ws_floats(uint32_t n, uint32_t heads, uint32_t kv_chunks) {
    return jc::attn_ws_floats(n, heads, kv_chunks);
}

size_t jc_attention_counters(uint32_t n, uint32_t heads) { return jc::attn_counters(n, heads); }

int jc_persist_tile(uint32_t m, uint32_t n, uint32_t k, uint32_t epi, uint32_t grid) {
    return (int)jc::persist_tile_width(m, n, k, epi, grid ? grid : 1);
}

double jc_gemm_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid) {
    if ((bn != 32 && bn != 64 && bn != 128 && bn != 256) || n % (uint32_t)bn) return -1.0;
    return jc::gemm_phase_us(m, n, k, bn, grid ? grid : 1);
}

double jc_persist_phase_us(uint32_t m, uint32_t n, uint32_t k, int bn, uint32_t grid) {
    if ((bn != 32 && bn != 64) || n % (uint32_t)bn) return -1.0;
    return jc::persist_phase_us(m, n, k, bn, grid ? grid : 1);
}

void jc_persist_tile_policy(int *bn) {
    if (!bn) return;
    if (*bn == 0 || *bn == 32 || *bn == 64)
        jc::swap_persist_tile_policy(bn);
    else
        *bn = -1;  // not a policy: nothing changed
}

void jc_gemm_tile_rows(int *rows) {
    if (rows && (*rows == 0 || *rows == 64 || *rows == 128)) jc::swap_gemm_tile_rows(rows);
}

void jc_gemm_pair_policy(int *policy) {
    if (!policy) return;
    if (*policy >= -1 && *policy <= 1)
        jc::swap_gemm_pair_policy(policy);
    else
        *policy = -2;  // not a policy: nothing changed
}

void jc_attention_tc_min(uint32_t *global_min, uint32_t *window_min) {
    if (global_min && window_min) jc::swap_attn_tc_min(global_min, window_min);
}

int jc_attention(const uint16_t *qkv, uint16_t *o, uint32_t n, uint32_t heads, uint32_t window,
                 uint32_t kv_chunks, float *ws, uint32_t *counters, void *stream) {
    return guarded(nullptr, 0, [&]() -> int {
        jc::AttnArgs a;
        a.qkv = reinterpret_cast<const __half *>(qkv);
        a.o = reinterpret_cast<__half *>(o);
        a.n = n;
        a.heads = heads;
        a.window = window;
        if (kv_chunks == 0) {
            int dev = 0, sms = 148;
            if (cudaGetDevice(&dev) == cudaSuccess)
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            kv_chunks = jc::choose_kv_chunks(n, heads, window, sms);
            if (!ws || !counters) kv_chunks = 1;
        }
        a.kv_chunks = kv_chunks;
        a.ws = ws;
        a.counters = counters;
        return jc::launch_attention(a, (cudaStream_t)stream, true) ? 0 : -1;
    });
}

int jc_embed(const uint32_t *ids, uint32_t n, const uint16_t *table, const float *gamma,
             uint32_t d, float eps, uint16_t *x, float *stats, void *stream) {
    return guarded(nullptr, 0, [&]() -> int {
        return jc::launch_embed(ids, n, reinterpret_cast<const __half *>(table), gamma, d, eps,
                                reinterpret_cast<__half *>(x), stats, (cudaStream_t)stream, true)
                   ? 0
                   : -1;
    });
}

int jc_norm_add(const uint16_t *x, uint32_t n, uint32_t d, const float *gamma, const float *add,
                float eps, uint16_t *out, float *stats, void *stream) {
    return guarded(nullptr, 0, [&]() -> int {
        return jc::launch_norm_add(reinterpret_cast<const __half *>(x), n, d, gamma, add, eps,
                                   reinterpret_cast<__half *>(out), stats, (cudaStream_t)stream,
                                   true)
                   ? 0
                   : -1;
    });
}

int jc_score(const uint16_t *y, uint32_t d, const uint16_t *w, float b, const uint32_t *markers,
             uint32_t k, float *logits, void *stream) {
    return guarded(nullptr, 0, [&]() -> int {
        return jc::launch_score(reinterpret_cast<const __half *>(y), d,
                                reinterpret_cast<const __half *>(w), b, markers, k, logits,
                                (cudaStream_t)stream, true)
                   ? 0
                   : -1;
    });
}

// ------------------------------------------------------------------------------------------
// host prep

void jc_prep_fold_layernorm(const float *w, const float *gamma, uint32_t out, uint32_t k,
                            uint16_t *w16, float *colsum) {
    jc::fold_layernorm(w, gamma, out, k, w16, colsum);
}

void jc_prep_fold_layernorm_bias(const float *w, const float *gamma, const float *beta,
                                 const float *b, uint32_t out, uint32_t k, uint16_t *w16,
                                 float *colsum, float *bias) {
    jc::fold_layernorm_bias(w, gamma, beta, b, out, k, w16, colsum, bias);
}

void jc_prep_interleave_geglu_f16(const uint16_t *w, uint32_t n, uint32_t k, uint16_t *out) {
    jc::interleave_geglu(w, n, k, out);
}

void jc_prep_interleave_geglu_f32(const float *w, uint32_t n, uint32_t k, float *out) {
    jc::interleave_geglu(w, n, k, out);
}

void jc_prep_rope_table(float theta, uint32_t n, float *out) { jc::rope_table(theta, n, out); }

void jc_prep_rope_gemm(const float *table, uint32_t m, float *out) {
    jc::rope_table_gemm(table, m, m, out);
}

}  // extern "C"
