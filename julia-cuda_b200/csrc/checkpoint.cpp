// Checkpoint directories (the reference's src/checkpoint.rs:27-62 and the tensors
// src/weights.rs:143-238 prepares): model.safetensors + encoder/config.json + julia_config.json.
//
// The reference parses these with julia-rs (`ModelConfig::load`, `safetensors::parse_header`),
// which is not available here, so the tensor names follow the public layouts they come from:
//   - the encoder is Hugging Face ModernBERT (`<prefix>embeddings.tok_embeddings.weight`,
//     `<prefix>layers.{i}.attn.Wqkv.weight`, ..., `<prefix>final_norm.weight`), the prefix found by
//     probing "model.", "encoder.model.", "encoder." and "" (or set in jc_names.json);
//   - the head layers are torch.nn.TransformerEncoderLayer's names (`head.layers.{i}.norm1.weight`,
//     `head.layers.{i}.self_attn.in_proj_weight`, ..., `head.layers.{i}.linear2.bias`), the type
//     embedding `type_emb.weight` and the scorer `scorer.{norm,lin1,lin2}.{weight,bias}`: the
//     fields the reference's HeadLayer / Scorer read (src/weights.rs:60-105), under a documented
//     default that an optional jc_names.json overrides tensor by tensor ({"encoder_prefix": "...",
//     "names": {"<default name>": "<name in the file>"}}).
// Shapes are checked against the config; head_ff, scorer_hidden, the question-type count and the
// head layer count come from the config files when they hold them and from the tensors' shapes
// otherwise. Tensors may be F32, F16 or BF16.
#include "checkpoint.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

#include "model.h"

namespace jc {
namespace {

// ---------------------------------------------------------------------------------------------
// a small JSON reader: objects, arrays, strings (with escapes), numbers, true / false / null

struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json *get(const std::string &k) const {
        if (kind != OBJ) return nullptr;
        for (const auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
   public:
    explicit JsonParser(const std::string &text) : s_(text), p_(s_.c_str()), end_(p_ + s_.size()) {}
    bool parse(Json *out, std::string *why) {
        if (!value(*out, 0)) {
            *why = err_;
            return false;
        }
        ws();
        if (p_ != end_) {
            *why = "trailing characters after the JSON value";
            return false;
        }
        return true;
    }

   private:
    std::string s_;
    const char *p_, *end_;
    std::string err_;

    bool fail(const char *m) {
        if (err_.empty()) err_ = m;
        return false;
    }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) p_++;
    }
    bool lit(const char *w) {
        const size_t n = strlen(w);
        if ((size_t)(end_ - p_) < n || strncmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string &s, uint32_t cp) {
        if (cp < 0x80) {
            s += (char)cp;
        } else if (cp < 0x800) {
            s += (char)(0xC0 | (cp >> 6));
            s += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18));
            s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(uint32_t *v) {
        if (end_ - p_ < 4) return fail("short \\u escape");
        *v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p_++;
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') *v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') *v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string &out) {
        p_++;  // the opening quote
        while (p_ < end_ && *p_ != '"') {
            if (*p_ != '\\') {
                out += *p_++;
                continue;
            }
            if (++p_ >= end_) return fail("unterminated escape");
            const char e = *p_++;
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        uint32_t lo;
                        if (!hex4(&lo)) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: return fail("bad escape in a JSON string");
            }
        }
        if (p_ >= end_) return fail("unterminated JSON string");
        p_++;
        return true;
    }
    bool value(Json &v, int depth) {
        if (depth > 64) return fail("JSON nested too deeply");
        ws();
        if (p_ >= end_) return fail("unexpected end of JSON");
        const char c = *p_;
        if (c == '{') {
            v.kind = Json::OBJ;
            p_++;
            ws();
            if (p_ < end_ && *p_ == '}') {
                p_++;
                return true;
            }
            while (true) {
                ws();
                if (p_ >= end_ || *p_ != '"') return fail("expected a key in a JSON object");
                std::string key;
                if (!string(key)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return fail("expected ':' in a JSON object");
                p_++;
                v.obj.emplace_back(std::move(key), Json());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    p_++;
                    return true;
                }
                return fail("expected ',' or '}' in a JSON object");
            }
        }
        if (c == '[') {
            v.kind = Json::ARR;
            p_++;
            ws();
            if (p_ < end_ && *p_ == ']') {
                p_++;
                return true;
            }
            while (true) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    p_++;
                    return true;
                }
                return fail("expected ',' or ']' in a JSON array");
            }
        }
        if (c == '"') {
            v.kind = Json::STR;
            return string(v.str);
        }
        if (lit("true")) {
            v.kind = Json::BOOL;
            v.b = true;
            return true;
        }
        if (lit("false")) {
            v.kind = Json::BOOL;
            return true;
        }
        if (lit("null")) return true;
        char *e = nullptr;
        v.num = strtod(p_, &e);  // the text is NUL-terminated (a std::string)
        if (e == p_) return fail("bad JSON value");
        v.kind = Json::NUM;
        p_ = e;
        return true;
    }
};

bool read_text(const std::string &path, std::string *out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    *out = ss.str();
    return true;
}

bool read_json(const std::string &path, Json *out, bool required, std::string *why) {
    std::string text;
    if (!read_text(path, &text)) {
        if (required) *why = "cannot read " + path;
        return !required;
    }
    std::string e;
    if (!JsonParser(text).parse(out, &e)) {
        *why = path + ": " + e;
        return false;
    }
    return true;
}

bool num_of(const Json &j, const char *key, double *v) {
    const Json *x = j.get(key);
    if (!x || x->kind != Json::NUM) return false;
    *v = x->num;
    return true;
}

// ---------------------------------------------------------------------------------------------
// the tensors of the raw format, in its order, with their default names and shapes

struct Entry {
    std::string name;            // default name (the encoder's without its prefix)
    bool encoder = false;        // carries the encoder prefix
    std::vector<uint64_t> shape;
    Span span;
};

std::vector<Entry> entries(const jc_model_config &c) {
    const RawLayout L = raw_layout(c);
    const uint64_t D = c.d_model, I = c.inter, F = c.head_ff, S = c.scorer_hidden;
    std::vector<Entry> out;
    auto add = [&](std::string name, bool enc, std::vector<uint64_t> shape, Span sp) {
        out.push_back(Entry{std::move(name), enc, std::move(shape), sp});
    };
    add("embeddings.tok_embeddings.weight", true, {(uint64_t)c.vocab, D}, L.tok_emb);
    add("embeddings.norm.weight", true, {D}, L.emb_norm);
    for (int l = 0; l < c.n_layers; l++) {
        const std::string p = "layers." + std::to_string(l) + ".";
        if (l > 0) add(p + "attn_norm.weight", true, {D}, L.attn_norm[l]);
        add(p + "attn.Wqkv.weight", true, {3 * D, D}, L.wqkv[l]);
        add(p + "attn.Wo.weight", true, {D, D}, L.wo[l]);
        add(p + "mlp_norm.weight", true, {D}, L.mlp_norm[l]);
        add(p + "mlp.Wi.weight", true, {2 * I, D}, L.wi[l]);
        add(p + "mlp.Wo.weight", true, {D, I}, L.wo_mlp[l]);
    }
    add("final_norm.weight", true, {D}, L.final_norm);
    add("type_emb.weight", false, {(uint64_t)c.n_qtypes, D}, L.type_emb);
    for (int l = 0; l < c.n_head_layers; l++) {
        const std::string p = "head.layers." + std::to_string(l) + ".";
        add(p + "norm1.weight", false, {D}, L.h_norm1_w[l]);
        add(p + "norm1.bias", false, {D}, L.h_norm1_b[l]);
        add(p + "self_attn.in_proj_weight", false, {3 * D, D}, L.h_in_w[l]);
        add(p + "self_attn.in_proj_bias", false, {3 * D}, L.h_in_b[l]);
        add(p + "self_attn.out_proj.weight", false, {D, D}, L.h_out_w[l]);
        add(p + "self_attn.out_proj.bias", false, {D}, L.h_out_b[l]);
        add(p + "norm2.weight", false, {D}, L.h_norm2_w[l]);
        add(p + "norm2.bias", false, {D}, L.h_norm2_b[l]);
        add(p + "linear1.weight", false, {F, D}, L.h_l1_w[l]);
        add(p + "linear1.bias", false, {F}, L.h_l1_b[l]);
        add(p + "linear2.weight", false, {D, F}, L.h_l2_w[l]);
        add(p + "linear2.bias", false, {D}, L.h_l2_b[l]);
    }
    add("scorer.norm.weight", false, {D}, L.s_norm_w);
    add("scorer.norm.bias", false, {D}, L.s_norm_b);
    add("scorer.lin1.weight", false, {S, D}, L.s_lin1_w);
    add("scorer.lin1.bias", false, {S}, L.s_lin1_b);
    add("scorer.lin2.weight", false, {1, S}, L.s_lin2_w);
    add("scorer.lin2.bias", false, {1}, L.s_lin2_b);
    return out;
}

// ---------------------------------------------------------------------------------------------
// safetensors: 8-byte little-endian header length, a JSON header {name: {dtype, shape,
// data_offsets: [begin, end)}}, then the data section

struct TensorInfo {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;
};

// A read-only mapping of a whole file.
class Mapped {
   public:
    ~Mapped() {
        if (p_ && p_ != MAP_FAILED) munmap(p_, n_);
        if (fd_ >= 0) close(fd_);
    }
    bool open(const std::string &path) {
        fd_ = ::open(path.c_str(), O_RDONLY);
        if (fd_ < 0) return false;
        struct stat st;
        if (fstat(fd_, &st) != 0 || st.st_size < 8) return false;
        n_ = (size_t)st.st_size;
        p_ = mmap(nullptr, n_, PROT_READ, MAP_PRIVATE, fd_, 0);
        return p_ != MAP_FAILED;
    }
    const uint8_t *data() const { return static_cast<const uint8_t *>(p_); }
    size_t size() const { return n_; }

   private:
    int fd_ = -1;
    void *p_ = nullptr;
    size_t n_ = 0;
};

size_t dtype_bytes(const std::string &d) {
    if (d == "F32") return 4;
    if (d == "F16" || d == "BF16") return 2;
    return 0;
}

float bf16_value(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

uint16_t bf16_bits(float x) {  // round to nearest even
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void convert(const uint8_t *src, const std::string &dtype, size_t n, float *dst) {
    if (dtype == "F32") {
        std::memcpy(dst, src, n * 4);
    } else if (dtype == "F16") {
        for (size_t i = 0; i < n; i++) {
            uint16_t h;
            std::memcpy(&h, src + 2 * i, 2);
            dst[i] = f16_value(h);
        }
    } else {
        for (size_t i = 0; i < n; i++) {
            uint16_t h;
            std::memcpy(&h, src + 2 * i, 2);
            dst[i] = bf16_value(h);
        }
    }
}

std::string shape_str(const std::vector<uint64_t> &s) {
    std::string o = "[";
    for (size_t i = 0; i < s.size(); i++) o += (i ? ", " : "") + std::to_string(s[i]);
    return o + "]";
}

}  // namespace

bool has_checkpoint(const std::string &dir) {
    struct stat st;
    return stat((dir + "/model.safetensors").c_str(), &st) == 0;
}

bool read_checkpoint(const std::string &dir, jc_model_config *cfg, std::vector<float> *raw,
                     std::string *why) {
    // --- the tensor index
    Mapped file;
    const std::string st_path = dir + "/model.safetensors";
    if (!file.open(st_path)) {
        *why = "cannot read " + st_path;
        return false;
    }
    uint64_t hlen = 0;
    std::memcpy(&hlen, file.data(), 8);
    if (hlen > file.size() - 8) {
        *why = "model.safetensors: header length " + std::to_string(hlen) + " exceeds the file size";
        return false;
    }
    const size_t data_start = 8 + (size_t)hlen, data_len = file.size() - data_start;
    Json header;
    {
        std::string e;
        if (!JsonParser(std::string(reinterpret_cast<const char *>(file.data()) + 8, (size_t)hlen))
                 .parse(&header, &e) ||
            header.kind != Json::OBJ) {
            *why = "model.safetensors header: " + (e.empty() ? std::string("not a JSON object") : e);
            return false;
        }
    }
    std::map<std::string, TensorInfo> index;
    for (const auto &kv : header.obj) {
        if (kv.first == "__metadata__") continue;
        const Json &t = kv.second;
        const Json *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
        if (!dt || dt->kind != Json::STR || !sh || sh->kind != Json::ARR || !off ||
            off->kind != Json::ARR || off->arr.size() != 2) {
            *why = "model.safetensors: tensor " + kv.first + " has no dtype, shape or data_offsets";
            return false;
        }
        TensorInfo ti;
        ti.dtype = dt->str;
        for (const Json &d : sh->arr) ti.shape.push_back((uint64_t)d.num);
        ti.begin = (uint64_t)off->arr[0].num;
        ti.end = (uint64_t)off->arr[1].num;
        if (ti.begin > ti.end || ti.end > data_len) {
            *why = "model.safetensors: tensor " + kv.first + " lies outside the data section";
            return false;
        }
        index.emplace(kv.first, std::move(ti));
    }

    // --- name overrides and the encoder's prefix
    Json names;
    if (!read_json(dir + "/jc_names.json", &names, false, why)) return false;
    std::string prefix;
    bool have_prefix = false;
    if (const Json *p = names.get("encoder_prefix"); p && p->kind == Json::STR) {
        prefix = p->str;
        have_prefix = true;
    }
    const Json *overrides = names.get("names");
    auto actual = [&](const std::string &def, bool enc) {
        if (overrides)
            if (const Json *o = overrides->get(def); o && o->kind == Json::STR) return o->str;
        return enc ? prefix + def : def;
    };
    if (!have_prefix) {
        bool found = false;
        for (const char *p : {"model.", "encoder.model.", "encoder.", ""})
            if (index.count(std::string(p) + "embeddings.tok_embeddings.weight")) {
                prefix = p;
                found = true;
                break;
            }
        if (!found && !(overrides && overrides->get("embeddings.tok_embeddings.weight"))) {
            *why = "model.safetensors: no ModernBERT embeddings (embeddings.tok_embeddings.weight "
                   "under the prefix model., encoder.model., encoder. or none; set "
                   "encoder_prefix in jc_names.json)";
            return false;
        }
    }
    auto find = [&](const std::string &def, bool enc) -> const TensorInfo * {
        auto it = index.find(actual(def, enc));
        return it == index.end() ? nullptr : &it->second;
    };

    // --- the config: the encoder's Hugging Face config, the head / scorer's julia_config.json,
    // and what the tensors' shapes say
    Json enc, jul;
    if (!read_json(dir + "/encoder/config.json", &enc, true, why) ||
        !read_json(dir + "/julia_config.json", &jul, false, why))
        return false;
    jc_model_config c;
    julia_cuda_default_config(&c);
    double v;
    auto need = [&](const char *key, double *out) {
        if (num_of(enc, key, out)) return true;
        *why = "encoder/config.json has no " + std::string(key);
        return false;
    };
    if (!need("hidden_size", &v)) return false;
    c.d_model = (int32_t)v;
    if (!need("intermediate_size", &v)) return false;
    c.inter = (int32_t)v;
    if (!need("num_hidden_layers", &v)) return false;
    c.n_layers = (int32_t)v;
    if (!need("vocab_size", &v)) return false;
    c.vocab = (int32_t)v;
    c.n_heads = num_of(enc, "num_attention_heads", &v) ? (int32_t)v : c.d_model / 64;
    if (num_of(enc, "norm_eps", &v)) c.norm_eps = (float)v;
    if (num_of(enc, "local_attention", &v)) c.window = (int32_t)v / 2;  // a +-window/2 span
    if (num_of(enc, "global_attn_every_n_layers", &v)) c.global_every = (int32_t)v;
    if (num_of(enc, "max_position_embeddings", &v)) c.max_positions = (int32_t)v;
    if (num_of(enc, "global_rope_theta", &v)) c.theta_global = (float)v;
    if (num_of(enc, "local_rope_theta", &v)) c.theta_local = (float)v;
    // The head's layer count: julia_config.json, else the head layers present.
    if (num_of(jul, "head_layers", &v) || num_of(jul, "num_head_layers", &v)) {
        c.n_head_layers = (int32_t)v;
    } else {
        int hl = 0;
        while (hl < 16 && find("head.layers." + std::to_string(hl) + ".linear1.weight", false)) hl++;
        c.n_head_layers = hl;
    }
    // Widths: julia_config.json, else the shapes of the tensors that carry them.
    auto width = [&](const char *k1, const char *k2, const std::string &tensor, int32_t *dst) {
        if (num_of(jul, k1, &v) || num_of(jul, k2, &v)) {
            *dst = (int32_t)v;
        } else if (const TensorInfo *t = find(tensor, false); t && !t->shape.empty()) {
            *dst = (int32_t)t->shape[0];
        }
    };
    width("head_ff", "dim_feedforward", "head.layers.0.linear1.weight", &c.head_ff);
    width("scorer_hidden", "scorer_dim", "scorer.lin1.weight", &c.scorer_hidden);
    width("n_qtypes", "num_qtypes", "type_emb.weight", &c.n_qtypes);
    if (num_of(jul, "head_eps", &v) || num_of(jul, "layer_norm_eps", &v)) c.head_eps = (float)v;
    if (!check_config(c, why)) {
        *why = "the checkpoint's config: " + *why;
        return false;
    }

    // --- the tensors, converted to f32 in the raw order
    raw->assign(raw_layout(c).total, 0.0f);
    for (const Entry &e : entries(c)) {
        const std::string name = actual(e.name, e.encoder);
        auto it = index.find(name);
        if (it == index.end()) {
            *why = "model.safetensors has no tensor " + name;
            return false;
        }
        const TensorInfo &t = it->second;
        const size_t es = dtype_bytes(t.dtype);
        if (!es) {
            *why = "tensor " + name + ": dtype " + t.dtype + " (F32, F16 or BF16 only)";
            return false;
        }
        uint64_t count = 1;
        for (uint64_t d : t.shape) count *= d;
        // A [1, S] vector may be stored as [S] and a [S] one as [1, S].
        std::vector<uint64_t> got = t.shape, want = e.shape;
        while (got.size() > 1 && got[0] == 1) got.erase(got.begin());
        while (want.size() > 1 && want[0] == 1) want.erase(want.begin());
        if (got != want || count != e.span.len) {
            *why = "tensor " + name + ": shape " + shape_str(t.shape) + ", the config wants " +
                   shape_str(e.shape);
            return false;
        }
        if (t.end - t.begin != count * es) {
            *why = "tensor " + name + ": its data is not " + std::to_string(count * es) + " bytes";
            return false;
        }
        convert(file.data() + data_start + t.begin, t.dtype, count, raw->data() + e.span.off);
    }
    *cfg = c;
    return true;
}

bool write_checkpoint(const std::string &dir, const jc_model_config &c, const float *raw,
                      int dtype, std::string *why) {
    if (!check_config(c, why)) return false;
    if (dtype < 0 || dtype > 2) {
        *why = "dtype must be 0 (F32), 1 (F16) or 2 (BF16)";
        return false;
    }
    const char *dname = dtype == 0 ? "F32" : dtype == 1 ? "F16" : "BF16";
    const size_t es = dtype == 0 ? 4 : 2;
    const std::vector<Entry> es_list = entries(c);
    std::string h = "{\"__metadata__\":{\"format\":\"pt\"}";
    uint64_t at = 0;
    for (const Entry &e : es_list) {
        const uint64_t bytes = e.span.len * es;
        h += ",\"" + std::string(e.encoder ? "model." : "") + e.name + "\":{\"dtype\":\"" + dname +
             "\",\"shape\":[";
        for (size_t i = 0; i < e.shape.size(); i++) h += (i ? "," : "") + std::to_string(e.shape[i]);
        h += "],\"data_offsets\":[" + std::to_string(at) + "," + std::to_string(at + bytes) + "]}";
        at += bytes;
    }
    h += "}";
    while ((8 + h.size()) % 8) h += ' ';  // the data section 8-byte aligned
    mkdir(dir.c_str(), 0755);
    mkdir((dir + "/encoder").c_str(), 0755);
    std::ofstream f(dir + "/model.safetensors", std::ios::binary);
    const uint64_t hlen = h.size();
    f.write(reinterpret_cast<const char *>(&hlen), 8);
    f.write(h.data(), (std::streamsize)h.size());
    std::vector<uint8_t> buf;
    for (const Entry &e : es_list) {
        const float *src = raw + e.span.off;
        buf.resize(e.span.len * es);
        for (size_t i = 0; i < e.span.len; i++) {
            if (dtype == 0) {
                std::memcpy(&buf[4 * i], &src[i], 4);
            } else {
                const uint16_t b = dtype == 1 ? f16_bits(src[i]) : bf16_bits(src[i]);
                std::memcpy(&buf[2 * i], &b, 2);
            }
        }
        f.write(reinterpret_cast<const char *>(buf.data()), (std::streamsize)buf.size());
    }
    char num[64];
    std::string ej = "{\n  \"architectures\": [\"ModernBertModel\"],\n  \"model_type\": \"modernbert\"";
    ej += ",\n  \"hidden_size\": " + std::to_string(c.d_model);
    ej += ",\n  \"intermediate_size\": " + std::to_string(c.inter);
    ej += ",\n  \"num_hidden_layers\": " + std::to_string(c.n_layers);
    ej += ",\n  \"num_attention_heads\": " + std::to_string(c.n_heads);
    ej += ",\n  \"vocab_size\": " + std::to_string(c.vocab);
    snprintf(num, sizeof num, "%.9g", (double)c.norm_eps);
    ej += ",\n  \"norm_eps\": " + std::string(num);
    ej += ",\n  \"local_attention\": " + std::to_string(2 * c.window);
    ej += ",\n  \"global_attn_every_n_layers\": " + std::to_string(c.global_every);
    ej += ",\n  \"max_position_embeddings\": " + std::to_string(c.max_positions);
    snprintf(num, sizeof num, "%.9g", (double)c.theta_global);
    ej += ",\n  \"global_rope_theta\": " + std::string(num);
    snprintf(num, sizeof num, "%.9g", (double)c.theta_local);
    ej += ",\n  \"local_rope_theta\": " + std::string(num) + "\n}\n";
    std::string jj = "{\n  \"head_layers\": " + std::to_string(c.n_head_layers);
    jj += ",\n  \"head_ff\": " + std::to_string(c.head_ff);
    jj += ",\n  \"scorer_hidden\": " + std::to_string(c.scorer_hidden);
    jj += ",\n  \"n_qtypes\": " + std::to_string(c.n_qtypes);
    snprintf(num, sizeof num, "%.9g", (double)c.head_eps);
    jj += ",\n  \"head_eps\": " + std::string(num) + "\n}\n";
    std::ofstream fe(dir + "/encoder/config.json"), fj(dir + "/julia_config.json");
    fe << ej;
    fj << jj;
    if (!f || !fe || !fj) {
        *why = "cannot write the checkpoint to " + dir;
        return false;
    }
    return true;
}

}  // namespace jc
