// host_io.cpp - safetensors shards and config.json on the host.
#include "host_io.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace pc {

int64_t StTensor::numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
}

StDB::~StDB() {
    for (int fd : fds_) close(fd);
}

namespace {

// Minimal JSON reader for safetensors headers.
struct JP {
    const char *p, *e;
    void ws() { while (p < e && isspace((unsigned char)*p)) ++p; }
    bool lit(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
    bool str(std::string &out) {
        ws();
        if (p >= e || *p != '"') return false;
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) { ++p; out.push_back(*p == 'n' ? '\n' : *p); ++p; continue; }
            out.push_back(*p++);
        }
        if (p >= e) return false;
        ++p;
        return true;
    }
    bool num(int64_t &v) {
        ws();
        char *end = nullptr;
        v = strtoll(p, &end, 10);
        if (end == p) return false;
        p = end;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{') {
            ++p;
            if (lit('}')) return true;
            do { std::string k; if (!str(k) || !lit(':') || !skip()) return false; } while (lit(','));
            return lit('}');
        }
        if (*p == '[') {
            ++p;
            if (lit(']')) return true;
            do { if (!skip()) return false; } while (lit(','));
            return lit(']');
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        return true;
    }
};

StDtype parse_dtype(const std::string &s) {
    if (s == "F32") return ST_F32;
    if (s == "F16") return ST_F16;
    if (s == "BF16") return ST_BF16;
    if (s == "I32") return ST_I32;
    if (s == "I16") return ST_I16;
    if (s == "I8") return ST_I8;
    if (s == "U8") return ST_U8;
    if (s == "F64") return ST_F64;
    if (s == "BOOL") return ST_BOOL;
    return ST_UNKNOWN;
}

bool exists(const std::string &p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0;
}

}  // namespace

bool StDB::open_file(const std::string &path, std::string *err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { *err = "cannot open " + path; return false; }
    uint64_t hlen = 0;
    if (pread(fd, &hlen, 8, 0) != 8 || hlen > (1ull << 31)) { close(fd); *err = "bad header in " + path; return false; }
    std::string h(hlen, '\0');
    if (pread(fd, &h[0], hlen, 8) != (ssize_t)hlen) { close(fd); *err = "short header in " + path; return false; }
    const int64_t data0 = 8 + (int64_t)hlen;
    const int fi = (int)fds_.size();
    fds_.push_back(fd);
    JP jp{h.data(), h.data() + h.size()};
    if (!jp.lit('{')) { *err = "bad header json in " + path; return false; }
    if (jp.lit('}')) return true;
    do {
        std::string name;
        if (!jp.str(name) || !jp.lit(':')) { *err = "bad header json in " + path; return false; }
        if (name == "__metadata__") { if (!jp.skip()) return false; continue; }
        StTensor t;
        t.file = fi;
        if (!jp.lit('{')) { *err = "bad tensor entry " + name; return false; }
        do {
            std::string key;
            if (!jp.str(key) || !jp.lit(':')) return false;
            if (key == "dtype") {
                std::string d;
                if (!jp.str(d)) return false;
                t.dtype = parse_dtype(d);
            } else if (key == "shape") {
                if (!jp.lit('[')) return false;
                if (!jp.lit(']')) {
                    do { int64_t v; if (!jp.num(v)) return false; t.shape.push_back(v); } while (jp.lit(','));
                    if (!jp.lit(']')) return false;
                }
            } else if (key == "data_offsets") {
                int64_t a, b;
                if (!jp.lit('[') || !jp.num(a) || !jp.lit(',') || !jp.num(b) || !jp.lit(']')) return false;
                t.begin = data0 + a;
                t.end = data0 + b;
            } else if (!jp.skip()) {
                return false;
            }
        } while (jp.lit(','));
        if (!jp.lit('}')) return false;
        map_.emplace(name, t);  // first occurrence wins
    } while (jp.lit(','));
    return true;
}

const StTensor *StDB::find(const std::string &name) const {
    auto it = map_.find(name);
    return it == map_.end() ? nullptr : &it->second;
}

bool StDB::read(const StTensor &t, void *dst, int64_t bytes, int64_t offset) const {
    if (offset < 0 || offset + bytes > t.nbytes()) return false;
    char *d = static_cast<char *>(dst);
    int64_t done = 0;
    while (done < bytes) {
        const ssize_t n = pread(fds_[t.file], d + done, (size_t)(bytes - done), t.begin + offset + done);
        if (n <= 0) return false;
        done += n;
    }
    return true;
}

bool open_model_dir(StDB &db, const std::string &dir, std::string *err) {
    char p[1024];
    auto try_open = [&](const std::string &path) -> bool {
        if (!exists(path)) return true;
        return db.open_file(path, err);
    };
    if (!try_open(dir + "/dense.safetensors")) return false;
    if (!try_open(dir + "/model.safetensors")) return false;
    for (int i = 1; i <= 200; ++i) {
        bool found = false;
        for (int total = 2; total <= 200; ++total) {
            snprintf(p, sizeof p, "%s/model-%05d-of-%05d.safetensors", dir.c_str(), i, total);
            if (exists(p)) {
                if (!db.open_file(p, err)) return false;
                found = true;
                break;
            }
        }
        if (!found && i > 1) break;
    }
    if (const char *aux = getenv("MODEL_AUX")) {
        std::string list(aux);
        size_t s = 0;
        while (s <= list.size()) {
            size_t q = list.find(';', s);
            if (q == std::string::npos) q = list.size();
            std::string one = list.substr(s, q - s);
            if (!one.empty() && exists(one) && !db.open_file(one, err)) return false;
            s = q + 1;
        }
    }
    for (int i = 0; i < 200; ++i) {
        snprintf(p, sizeof p, "%s/model-%05d.safetensors", dir.c_str(), i);
        if (!try_open(p)) return false;
    }
    for (int i = 0; i < 50; ++i) {
        snprintf(p, sizeof p, "%s/experts-%02d.safetensors", dir.c_str(), i);
        if (!try_open(p)) return false;
    }
    if (db.n_tensors() == 0) { *err = "no tensors found in " + dir; return false; }
    return true;
}

// ---- config.json, json.h semantics ----------------------------------------
namespace {

const char *find_key(const std::string &js, const char *key) {
    const size_t kl = strlen(key);
    size_t pos = 0;
    while ((pos = js.find(key, pos)) != std::string::npos) {
        if (pos > 0 && js[pos - 1] == '"' && pos + kl < js.size() && js[pos + kl] == '"') {
            size_t q = pos + kl + 1;
            while (q < js.size() && isspace((unsigned char)js[q])) ++q;
            if (q < js.size() && js[q] == ':') return js.c_str() + q + 1;
        }
        ++pos;
    }
    return nullptr;
}

const char *skip_ws(const char *v) {
    while (v && *v && isspace((unsigned char)*v)) ++v;
    return v;
}

int j_int(const std::string &js, const char *key, int def) {
    const char *v = find_key(js, key);
    if (!v) return def;
    v = skip_ws(v);
    if (*v == 'n') return def;
    return atoi(v);
}

float j_float(const std::string &js, const char *key, float def) {
    const char *v = find_key(js, key);
    if (!v) return def;
    v = skip_ws(v);
    if (*v == 'n') return def;
    return (float)atof(v);
}

int j_bool(const std::string &js, const char *key, int def) {
    const char *v = find_key(js, key);
    if (!v) return def;
    v = skip_ws(v);
    if (*v == 't') return 1;
    if (*v == 'f') return 0;
    return def;
}

}  // namespace

bool load_config(const std::string &dir, pc_model_cfg *c, std::string *err) {
    FILE *f = fopen((dir + "/config.json").c_str(), "rb");
    if (!f) { *err = "cannot read " + dir + "/config.json"; return false; }
    std::string js;
    char buf[4096];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) js.append(buf, n);
    fclose(f);
    memset(c, 0, sizeof *c);
    c->hidden = j_int(js, "hidden_size", 2880);
    c->n_layers = j_int(js, "num_hidden_layers", 36);
    c->n_heads = j_int(js, "num_attention_heads", 64);
    c->n_kv_heads = j_int(js, "num_key_value_heads", 8);
    c->head_dim = j_int(js, "head_dim", 64);
    c->n_experts = j_int(js, "num_local_experts", 128);
    c->topk = j_int(js, "num_experts_per_tok", 4);
    c->intermediate = j_int(js, "intermediate_size", 2880);
    c->vocab = j_int(js, "vocab_size", 201088);
    c->ctx_len = j_int(js, "max_position_embeddings", 131072);
    c->sliding_window = j_int(js, "sliding_window", 128);
    c->eps = j_float(js, "rms_norm_eps", 1e-5f);
    c->theta = j_float(js, "rope_theta", 150000.0f);
    c->rope_factor = j_float(js, "factor", 1.0f);
    c->rope_beta_fast = j_float(js, "beta_fast", 32.0f);
    c->rope_beta_slow = j_float(js, "beta_slow", 1.0f);
    c->rope_original_ctx = j_int(js, "original_max_position_embeddings", c->ctx_len);
    c->rope_truncate = j_bool(js, "truncate", 1);
    c->swiglu_limit = j_float(js, "swiglu_limit", 7.0f);
    c->swiglu_alpha = 1.702f;
    c->routed_scale = j_float(js, "routed_scaling_factor", 1.0f);
    if (c->n_layers <= 0 || c->n_layers > 256) { *err = "num_hidden_layers out of range"; return false; }
    // layer_types (picchio.c:389-409): "full" anywhere in the name -> full
    std::vector<std::string> types;
    if (const char *v = find_key(js, "layer_types")) {
        v = skip_ws(v);
        if (*v == '[') {
            ++v;
            while (*v && *v != ']' && types.size() < 128) {
                v = skip_ws(v);
                if (*v == '"') {
                    ++v;
                    std::string s;
                    while (*v && *v != '"' && s.size() < 63) {
                        if (*v == '\\' && v[1]) ++v;
                        s.push_back(*v++);
                    }
                    if (*v == '"') ++v;
                    types.push_back(s);
                }
                while (*v && *v != '"' && *v != ']') ++v;
            }
        }
    }
    for (int i = 0; i < c->n_layers; ++i) {
        if (!types.empty())
            c->layer_type[i] = types[i % types.size()].find("full") != std::string::npos ? 1 : 0;
        else
            c->layer_type[i] = i % 2;
    }
    return true;
}

}  // namespace pc
