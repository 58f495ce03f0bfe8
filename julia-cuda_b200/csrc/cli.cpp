// julia-cuda: the command-line front end (the reference's src/main.rs and src/serve.rs), built on
// the library's public C ABI alone (include/julia_cuda.h).
//
//   julia-cuda [MODEL_DIR | --random SEED] [--max-length N] [--head-length N] [--layer-fused |
//              --mode M] [--pack ROWS] [--set KEY=VALUE ...] < requests.jsonl > results.jsonl
//   julia-cuda  MODEL_DIR | --random SEED  --check | --time
//
// Without a model it checks that the kernels load and run on GPU 0 (a tiny seeded model, one
// request). With one it answers the requests on stdin, one JSON object per line, in order, with
// one result line each, and reports latency percentiles on stderr (src/serve.rs:22-115). The
// reference tokenizes text requests with julia-rs, which is not available here, so a request holds
// token ids: {"ids": [...], "markers": [...], "qtype": 0 | 1 | 2 or "choice" | "score" | "noul"}.
// A result holds the marker logits, their softmax ("probabilities", what the reference's
// tools/score.py reads), the argmax marker ("choice"), "truncated": false (requests longer than
// --max-length are rejected, not truncated) and "gpu_ms" (embed to logits).
//   --check  runs seeded sample requests in all three execution modes (per-step kernels, one
//            persistent launch per layer, one for the whole model) and requires finite logits,
//            the same argmax and logits within 2e-3 of the per-step kernels' (the f32 reference
//            comparisons live in the test suite, which has the CPU oracle).
//   --time   measures each mode's GPU time per request (CUDA events, embed to logits) on the
//            sample requests after warm-up.
//   --random SEED   seeded synthetic weights (julia_cuda_init_random) instead of a directory;
//   --set KEY=VALUE overrides a field of the benchmark model's config for them (d_model, inter,
//            n_layers, vocab, head_ff, scorer_hidden, n_head_layers, max_positions, ...).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <random>
#include <string>
#include <vector>

#include "../../include/julia_cuda.h"

namespace {

const char *USAGE =
    "usage: julia-cuda [MODEL_DIR | --random SEED [--set KEY=VALUE ...]] [--max-length N]\n"
    "                  [--head-length N] [--layer-fused | --mode 0|1|2] [--pack ROWS]\n"
    "                  < requests.jsonl > results.jsonl\n"
    "       julia-cuda MODEL_DIR | --random SEED  --check | --time\n"
    "  Without a model, checks that the kernels load and run on GPU 0. With one, answers the\n"
    "  requests on stdin ({\"ids\": [...], \"markers\": [...], \"qtype\": 0}), one JSON line each, and\n"
    "  reports latency on stderr. MODEL_DIR holds model.safetensors + encoder/config.json +\n"
    "  julia_config.json (or jc_config.bin + jc_weights.f32). --mode 1 (--layer-fused) runs each\n"
    "  encoder layer as one persistent launch, --mode 2 the whole model as one. --pack packs\n"
    "  consecutive requests into forwards of up to ROWS tokens.\n"
    "  --check runs sample requests in all three modes and compares them; --time measures each\n"
    "  mode's GPU time per request.\n";

struct Request {
    std::vector<uint32_t> ids, markers;
    uint32_t qtype = 0;
};

// --- a reader for one request line: a flat JSON object of number arrays, numbers and strings
class Line {
   public:
    explicit Line(const std::string &s) : p_(s.c_str()), end_(s.c_str() + s.size()) {}
    bool parse(Request *r, std::string *why) {
        ws();
        if (!eat('{')) return fail(why, "a request is a JSON object");
        ws();
        if (eat('}')) return fail(why, "empty request");
        while (true) {
            std::string key;
            ws();
            if (!str(&key)) return fail(why, "expected a key");
            ws();
            if (!eat(':')) return fail(why, "expected ':'");
            ws();
            if (key == "ids" || key == "markers") {
                std::vector<uint32_t> &v = key == "ids" ? r->ids : r->markers;
                if (!array(&v)) return fail(why, ("bad array \"" + key + "\"").c_str());
            } else if (key == "qtype") {
                std::string s;
                double d;
                if (*p_ == '"') {
                    if (!str(&s)) return fail(why, "bad qtype");
                    if (s == "choice") r->qtype = 0;
                    else if (s == "score") r->qtype = 1;
                    else if (s == "noul") r->qtype = 2;
                    else return fail(why, "qtype must be choice, score or noul (or 0, 1, 2)");
                } else if (number(&d) && d >= 0 && d == std::floor(d)) {
                    r->qtype = (uint32_t)d;
                } else {
                    return fail(why, "bad qtype");
                }
            } else if (!skip()) {
                return fail(why, ("bad value of \"" + key + "\"").c_str());
            }
            ws();
            if (eat(',')) continue;
            if (eat('}')) break;
            return fail(why, "expected ',' or '}'");
        }
        ws();
        if (p_ != end_) return fail(why, "trailing characters");
        if (r->ids.empty()) return fail(why, "no \"ids\"");
        return true;
    }

   private:
    const char *p_, *end_;
    static bool fail(std::string *why, const char *m) {
        *why = m;
        return false;
    }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\r' || *p_ == '\n')) p_++;
    }
    bool eat(char c) {
        if (p_ < end_ && *p_ == c) {
            p_++;
            return true;
        }
        return false;
    }
    bool str(std::string *out) {
        if (!eat('"')) return false;
        while (p_ < end_ && *p_ != '"') {
            if (*p_ == '\\') {
                if (++p_ >= end_) return false;
            }
            *out += *p_++;
        }
        return eat('"');
    }
    bool number(double *d) {
        char *e = nullptr;
        *d = strtod(p_, &e);  // the line is NUL-terminated (a std::string)
        if (e == p_ || e > end_) return false;
        p_ = e;
        return true;
    }
    bool array(std::vector<uint32_t> *v) {
        if (!eat('[')) return false;
        ws();
        if (eat(']')) return true;
        while (true) {
            ws();
            double d;
            if (!number(&d) || d < 0 || d > 4294967295.0 || d != std::floor(d)) return false;
            v->push_back((uint32_t)d);
            ws();
            if (eat(',')) continue;
            return eat(']');
        }
    }
    bool skip() {  // any other value, nested
        int depth = 0;
        bool in_str = false;
        for (; p_ < end_; p_++) {
            const char c = *p_;
            if (in_str) {
                if (c == '\\') p_++;
                else if (c == '"') in_str = false;
                continue;
            }
            if (c == '"') in_str = true;
            else if (c == '[' || c == '{') depth++;
            else if (c == ']' || c == '}') {
                if (depth == 0) return true;
                depth--;
            } else if (c == ',' && depth == 0) return true;
        }
        return depth == 0;
    }
};

double now_ms() {
    return std::chrono::duration<double, std::milli>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

std::string pct(std::vector<double> v) {
    if (v.empty()) return "-";
    std::sort(v.begin(), v.end());
    auto at = [&](double p) { return v[(size_t)std::lround((double)(v.size() - 1) * p)]; };
    double sum = 0;
    for (double x : v) sum += x;
    char buf[200];
    snprintf(buf, sizeof buf, "mean %.3f, p50 %.3f, p90 %.3f, p99 %.3f, max %.3f ms",
             sum / (double)v.size(), at(0.5), at(0.9), at(0.99), at(1.0));
    return buf;
}

bool set_field(jc_model_config *c, const std::string &kv) {
    const size_t eq = kv.find('=');
    if (eq == std::string::npos) return false;
    const std::string k = kv.substr(0, eq);
    const double v = atof(kv.c_str() + eq + 1);
    int32_t *ints[] = {&c->d_model, &c->inter, &c->n_layers, &c->vocab, &c->head_ff,
                       &c->scorer_hidden, &c->n_head_layers, &c->global_every, &c->window,
                       &c->max_positions, &c->n_qtypes};
    const char *names[] = {"d_model", "inter", "n_layers", "vocab", "head_ff", "scorer_hidden",
                           "n_head_layers", "global_every", "window", "max_positions", "n_qtypes"};
    for (size_t i = 0; i < sizeof names / sizeof names[0]; i++)
        if (k == names[i]) {
            *ints[i] = (int32_t)v;
            if (k == "d_model") c->n_heads = c->d_model / 64;
            return true;
        }
    if (k == "norm_eps") c->norm_eps = (float)v;
    else if (k == "head_eps") c->head_eps = (float)v;
    else if (k == "theta_global") c->theta_global = (float)v;
    else if (k == "theta_local") c->theta_local = (float)v;
    else return false;
    return true;
}

// Seeded sample requests (the reference's --check / --time run its sample requests): 293 tokens
// (the benchmark's length) and the longest the engine takes, four markers each.
std::vector<Request> samples(const jc_model_config &c, size_t max_length, size_t head_length) {
    std::vector<Request> out;
    std::mt19937_64 rng(293);
    for (size_t n : {std::min<size_t>(293, max_length), max_length}) {
        Request r;
        for (size_t i = 0; i < n; i++) r.ids.push_back((uint32_t)(rng() % (uint64_t)c.vocab));
        const size_t span = head_length && head_length < n ? head_length : n;
        for (size_t j = 0; j < 4 && j < span; j++) r.markers.push_back((uint32_t)(j * span / 4));
        out.push_back(r);
        if (n == max_length) break;
    }
    return out;
}

int run_batch(JcEngine *e, const std::vector<Request> &reqs, int mode, std::vector<float> *logits,
              std::vector<float> *gpu_ms, std::string *why) {
    std::vector<uint32_t> ids, mk, qt;
    std::vector<size_t> lens, nmk;
    for (const Request &r : reqs) {
        ids.insert(ids.end(), r.ids.begin(), r.ids.end());
        mk.insert(mk.end(), r.markers.begin(), r.markers.end());
        lens.push_back(r.ids.size());
        nmk.push_back(r.markers.size());
        qt.push_back(r.qtype);
    }
    logits->assign(std::max<size_t>(mk.size(), 1), 0.f);
    gpu_ms->assign(reqs.size(), 0.f);
    char err[1024] = {0};
    const int rc = julia_cuda_run(e, reqs.size(), ids.data(), lens.data(), mk.data(), nmk.data(),
                                  qt.data(), mode, logits->data(), gpu_ms->data(), err, sizeof err);
    if (rc != 0) *why = err;
    return rc;
}

int check(JcEngine *e, const std::vector<Request> &reqs) {
    std::vector<std::vector<float>> per_mode(3);
    for (int mode = 0; mode < 3; mode++) {
        std::vector<float> gpu_ms;
        std::string why;
        if (run_batch(e, reqs, mode, &per_mode[mode], &gpu_ms, &why) != 0) {
            fprintf(stderr, "check: mode %d: %s\n", mode, why.c_str());
            return 1;
        }
    }
    bool ok = true;
    size_t at = 0;
    for (size_t i = 0; i < reqs.size(); i++) {
        const size_t k = reqs[i].markers.size();
        double worst[3] = {0, 0, 0};
        size_t arg[3] = {0, 0, 0};
        for (int mode = 0; mode < 3; mode++) {
            for (size_t j = 0; j < k; j++) {
                const float v = per_mode[mode][at + j];
                if (!std::isfinite(v)) ok = false;
                if (v > per_mode[mode][at + arg[mode]]) arg[mode] = j;
                worst[mode] = std::max(worst[mode], (double)std::fabs(v - per_mode[0][at + j]));
            }
        }
        const bool same = arg[1] == arg[0] && arg[2] == arg[0];
        const bool close = worst[1] < 2e-3 && worst[2] < 2e-3;
        fprintf(stderr,
                "request %zu (%zu tokens): logits", i, reqs[i].ids.size());
        for (size_t j = 0; j < k; j++) fprintf(stderr, " %.5f", per_mode[0][at + j]);
        fprintf(stderr, "; layer-fused max |d| %.2e, whole-model max |d| %.2e, answers %s\n",
                worst[1], worst[2], same ? "agree" : "DIFFER");
        ok = ok && same && close;
        at += k;
    }
    fprintf(stderr, "check: %s\n", ok ? "ok" : "FAILED");
    return ok ? 0 : 1;
}

int time_modes(JcEngine *e, const std::vector<Request> &reqs) {
    const char *names[] = {"per-step kernels (CUDA graph + PDL)", "one persistent launch per layer",
                           "whole model, one persistent launch"};
    for (const Request &r : reqs) {
        for (int mode = 0; mode < 3; mode++) {
            std::vector<float> logits, ms;
            std::vector<double> all;
            std::string why;
            for (int i = 0; i < 5; i++)
                if (run_batch(e, {r}, mode, &logits, &ms, &why) != 0) {
                    fprintf(stderr, "time: %s\n", why.c_str());
                    return 1;
                }
            for (int i = 0; i < 50; i++) {
                if (run_batch(e, {r}, mode, &logits, &ms, &why) != 0) {
                    fprintf(stderr, "time: %s\n", why.c_str());
                    return 1;
                }
                all.push_back(ms[0]);
            }
            fprintf(stderr, "%zu tokens, %s (%d launches): GPU %s\n", r.ids.size(), names[mode],
                    julia_cuda_launches_per_forward(e, (uint32_t)r.ids.size(),
                                                    (uint32_t)r.markers.size(), mode),
                    pct(all).c_str());
        }
    }
    return 0;
}

int serve(JcEngine *e, int mode) {
    std::vector<std::pair<double, double>> stats;  // (wall ms, GPU ms)
    std::vector<size_t> tokens;
    std::string line;
    size_t lineno = 0;
    while (std::getline(std::cin, line)) {
        lineno++;
        if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
        const double t0 = now_ms();
        Request r;
        std::string why;
        if (!Line(line).parse(&r, &why)) {
            fprintf(stderr, "line %zu: %s\n", lineno, why.c_str());
            return 1;
        }
        std::vector<float> logits, ms;
        if (run_batch(e, {r}, mode, &logits, &ms, &why) != 0) {
            fprintf(stderr, "line %zu: %s\n", lineno, why.c_str());
            return 1;
        }
        const size_t k = r.markers.size();
        double mx = -INFINITY, sum = 0;
        size_t arg = 0;
        for (size_t j = 0; j < k; j++)
            if (logits[j] > mx) {
                mx = logits[j];
                arg = j;
            }
        std::vector<double> prob(k);
        for (size_t j = 0; j < k; j++) sum += prob[j] = std::exp((double)logits[j] - mx);
        std::string out = "{\"logits\": [";
        char num[64];
        for (size_t j = 0; j < k; j++) {
            snprintf(num, sizeof num, "%s%.9g", j ? ", " : "", (double)logits[j]);
            out += num;
        }
        out += "], \"probabilities\": [";
        for (size_t j = 0; j < k; j++) {
            snprintf(num, sizeof num, "%s%.9g", j ? ", " : "", prob[j] / sum);
            out += num;
        }
        snprintf(num, sizeof num, "%.6f", (double)ms[0]);
        out += "], \"choice\": " + (k ? std::to_string(arg) : std::string("null")) +
               ", \"truncated\": false, \"gpu_ms\": " + num + "}";
        std::cout << out << "\n";
        stats.emplace_back(now_ms() - t0, ms[0]);
        tokens.push_back(r.ids.size());
    }
    std::cout.flush();
    if (stats.empty()) {
        fprintf(stderr, "no requests\n");
        return 0;
    }
    size_t tsum = 0;
    for (size_t t : tokens) tsum += t;
    fprintf(stderr, "%zu requests, %zu tokens on average (%zu-%zu); the first took %.1f ms (wall)\n",
            stats.size(), tsum / tokens.size(), *std::min_element(tokens.begin(), tokens.end()),
            *std::max_element(tokens.begin(), tokens.end()), stats[0].first);
    if (stats.size() > 1) {
        std::vector<double> wall, gpu;
        for (size_t i = 1; i < stats.size(); i++) {
            wall.push_back(stats[i].first);
            gpu.push_back(stats[i].second);
        }
        fprintf(stderr, "  per request, wall (parse, upload, run, download): %s\n", pct(wall).c_str());
        fprintf(stderr, "  per request, GPU (embed to logits):               %s\n", pct(gpu).c_str());
    }
    return 0;
}

}  // namespace

int main(int argc, char **argv) {
    std::string dir;
    bool random = false, do_check = false, do_time = false;
    uint64_t seed = 0;
    size_t max_length = 0, head_length = 0, pack = 0;
    int mode = 0;
    jc_model_config cfg;
    julia_cuda_default_config(&cfg);
    for (int i = 1; i < argc; i++) {
        const std::string a = argv[i];
        auto next = [&](const char *what) -> const char * {
            if (i + 1 >= argc) {
                fprintf(stderr, "%s needs a value\n%s", what, USAGE);
                exit(2);
            }
            return argv[++i];
        };
        if (a == "--check") do_check = true;
        else if (a == "--time") do_time = true;
        else if (a == "--layer-fused") mode = 1;
        else if (a == "--mode") mode = atoi(next("--mode"));
        else if (a == "--max-length") max_length = strtoull(next("--max-length"), nullptr, 10);
        else if (a == "--head-length") head_length = strtoull(next("--head-length"), nullptr, 10);
        else if (a == "--pack") pack = strtoull(next("--pack"), nullptr, 10);
        else if (a == "--random") {
            random = true;
            seed = strtoull(next("--random"), nullptr, 10);
        } else if (a == "--set") {
            if (!set_field(&cfg, next("--set"))) {
                fprintf(stderr, "--set: unknown field in %s\n", argv[i]);
                return 2;
            }
        } else if (a == "-h" || a == "--help") {
            fputs(USAGE, stdout);
            return 0;
        } else if (!a.empty() && a[0] != '-' && dir.empty()) {
            dir = a;
        } else {
            fprintf(stderr, "unknown argument %s\n%s", a.c_str(), USAGE);
            return 2;
        }
    }
    if (mode < 0 || mode > 2 || (random && !dir.empty())) {
        fputs(USAGE, stderr);
        return 2;
    }
    char err[1024] = {0};
    if (dir.empty() && !random) {
        // No model: the kernels load and run on GPU 0 (a tiny seeded model, one request).
        jc_model_config tiny = cfg;
        tiny.d_model = 128, tiny.n_heads = 2, tiny.inter = 128, tiny.n_layers = 3, tiny.vocab = 64;
        tiny.head_ff = 128, tiny.scorer_hidden = 64, tiny.max_positions = 128;
        JcEngine *e = julia_cuda_load_random(&tiny, 1, 128, 0, err, sizeof err);
        if (!e) {
            fprintf(stderr, "julia-cuda: %s\n", err);
            return 1;
        }
        std::vector<float> logits, ms;
        std::string why;
        Request r;
        for (uint32_t i = 0; i < 100; i++) r.ids.push_back(i % 64);
        r.markers = {0, 50, 99};
        const int rc = run_batch(e, {r}, 0, &logits, &ms, &why);
        char name[256] = {0};
        julia_cuda_device(e, name, sizeof name);
        julia_cuda_free(e);
        if (rc != 0) {
            fprintf(stderr, "julia-cuda: %s\n", why.c_str());
            return 1;
        }
        fprintf(stderr, "kernels (%s) load and run on %s\n", julia_cuda_tier(), name);
        return 0;
    }
    const double t0 = now_ms();
    JcEngine *e = nullptr;
    if (random) {
        e = julia_cuda_load_random(&cfg, seed, max_length, 0, err, sizeof err);
    } else {
        e = julia_cuda_load(dir.c_str(), max_length, err, sizeof err);
    }
    if (!e) {
        fprintf(stderr, "julia-cuda: %s\n", err);
        return 1;
    }
    size_t cap = 0;
    julia_cuda_engine_config(e, &cfg, &cap, nullptr, nullptr);
    char name[256] = {0};
    julia_cuda_device(e, name, sizeof name);
    fprintf(stderr, "model: %d layers, hidden %d, intermediate %d, %d head layers; %s; up to %zu "
            "tokens (%.0f ms to load)\n", cfg.n_layers, cfg.d_model, cfg.inter, cfg.n_head_layers,
            name, cap, now_ms() - t0);
    if (head_length) julia_cuda_set_head_length(e, head_length);
    if (pack && julia_cuda_set_packing(e, pack) != 0) {
        fprintf(stderr, "julia-cuda: --pack %zu is over --max-length\n", pack);
        julia_cuda_free(e);
        return 2;
    }
    int rc = 0;
    if (do_check || do_time) {
        const std::vector<Request> reqs = samples(cfg, cap, head_length);
        if (do_check) rc = check(e, reqs);
        if (rc == 0 && do_time) rc = time_modes(e, reqs);
    } else {
        rc = serve(e, mode);
    }
    julia_cuda_free(e);
    return rc;
}
