// g2_loader.cpp -- config.json and safetensors reading (host side of g2_open).
#include "g2_loader.h"

#include <cstring>

#include "gpt2b200.h"

namespace g2 {

static bool slurp(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    out.clear();
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

// First occurrence of "key", then ':', then a decimal integer (as the
// reference's json_get_int_any, main.c:272-287).
static bool json_int(const std::string &js, const char *key, int &out) {
    std::string pat = std::string("\"") + key + "\"";
    size_t p = js.find(pat);
    if (p == std::string::npos) return false;
    p = js.find(':', p + pat.size());
    if (p == std::string::npos) return false;
    ++p;
    while (p < js.size() && (js[p] == ' ' || js[p] == '\t')) ++p;
    out = atoi(js.c_str() + p);
    return true;
}

int load_config(const std::string &dir, ModelConfig &c, std::string &err) {
    std::string js;
    c = ModelConfig();
    if (slurp(dir + "/config.json", js)) {
        json_int(js, "n_layer", c.n_layer);
        json_int(js, "n_embd", c.n_embd);
        json_int(js, "n_head", c.n_head);
        if (!json_int(js, "n_positions", c.n_ctx)) json_int(js, "n_ctx", c.n_ctx);
        json_int(js, "vocab_size", c.vocab_size);
        int inner = 0;
        json_int(js, "n_inner", inner);
        c.ffn_dim = inner > 0 ? inner : 4 * c.n_embd;
    }
    if (c.n_layer <= 0 || c.n_embd <= 0 || c.n_head <= 0 || c.vocab_size <= 0 || c.ffn_dim <= 0) {
        err = "config.json: non-positive dimension";
        return G2_ERR_FORMAT;
    }
    if (c.n_embd != c.n_head * 64) {
        err = "config.json: head size must be 64 (n_embd = 64 * n_head)";
        return G2_ERR_FORMAT;
    }
    if (c.n_ctx <= 0 || c.n_ctx > 1024) {
        err = "config.json: n_ctx must be in 1..1024";
        return G2_ERR_FORMAT;
    }
    if (c.ffn_dim % 16 || c.n_embd % 16) {
        err = "config.json: n_embd and ffn must be multiples of 16";
        return G2_ERR_FORMAT;
    }
    c.padded_vocab = (c.vocab_size + 3) & ~3;
    return G2_OK;
}

// ---- safetensors: 8-byte little-endian header length, JSON header, data ----------
namespace {
struct Parser {
    const char *p, *end;
    bool ok = true;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool lit(char c) {
        ws();
        if (p < end && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    bool str(std::string &out) {
        ws();
        if (p >= end || *p != '"') return ok = false;
        ++p;
        out.clear();
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return ok = false;
                c = *p++;
                if (c == 'u') {   // keep \uXXXX escapes verbatim; tensor names are ASCII
                    out += "\\u";
                    continue;
                }
            }
            out += c;
        }
        if (p >= end) return ok = false;
        ++p;
        return true;
    }
    bool integer(int64_t &v) {
        ws();
        char *e = nullptr;
        long long x = strtoll(p, &e, 10);
        if (e == p || e > end) return ok = false;
        p = e;
        v = x;
        return true;
    }
    bool int_array(std::vector<int64_t> &v) {
        v.clear();
        if (!lit('[')) return ok = false;
        if (lit(']')) return true;
        do {
            int64_t x;
            if (!integer(x)) return false;
            v.push_back(x);
        } while (lit(','));
        return lit(']') || (ok = false);
    }
    bool skip() {
        ws();
        if (p >= end) return ok = false;
        if (*p == '"') {
            std::string s;
            return str(s);
        }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            ++p;
            if (lit(close)) return true;
            do {
                if (obj) {
                    std::string k;
                    if (!str(k) || !lit(':')) return ok = false;
                }
                if (!skip()) return false;
            } while (lit(','));
            return lit(close) || (ok = false);
        }
        while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
        return true;
    }
};
}  // namespace

SafeTensors::~SafeTensors() {
    if (fp_) fclose(fp_);
}

int SafeTensors::open(const std::string &path, std::string &err) {
    fp_ = fopen(path.c_str(), "rb");
    if (!fp_) {
        err = "cannot open " + path;
        return G2_ERR_IO;
    }
    fseeko(fp_, 0, SEEK_END);
    file_size_ = ftello(fp_);
    fseeko(fp_, 0, SEEK_SET);
    unsigned char lb[8];
    if (fread(lb, 1, 8, fp_) != 8) {
        err = "safetensors: cannot read header length";
        return G2_ERR_FORMAT;
    }
    uint64_t hl = 0;
    for (int i = 7; i >= 0; --i) hl = (hl << 8) | lb[i];
    if (hl == 0 || hl > (100ull << 20) || (int64_t)(8 + hl) > file_size_) {
        err = "safetensors: implausible header length";
        return G2_ERR_FORMAT;
    }
    std::string h(hl, '\0');
    if (fread(&h[0], 1, hl, fp_) != hl) {
        err = "safetensors: short header";
        return G2_ERR_FORMAT;
    }
    data_start_ = 8 + (int64_t)hl;
    Parser ps{h.data(), h.data() + h.size()};
    if (!ps.lit('{')) {
        err = "safetensors: header is not a JSON object";
        return G2_ERR_FORMAT;
    }
    if (!ps.lit('}')) {
        do {
            std::string key;
            if (!ps.str(key) || !ps.lit(':')) break;
            if (key == "__metadata__") {
                if (!ps.skip()) break;
                continue;
            }
            StTensor t;
            t.name = key;
            if (!ps.lit('{')) {
                ps.ok = false;
                break;
            }
            if (!ps.lit('}')) {
                do {
                    std::string f;
                    if (!ps.str(f) || !ps.lit(':')) break;
                    if (f == "dtype") {
                        std::string d;
                        if (!ps.str(d)) break;
                        t.dtype = d == "F32" ? ST_F32 : d == "F16" ? ST_F16 : d == "BF16" ? ST_BF16 : ST_OTHER;
                    } else if (f == "shape") {
                        if (!ps.int_array(t.shape)) break;
                    } else if (f == "data_offsets") {
                        std::vector<int64_t> o;
                        if (!ps.int_array(o) || o.size() != 2) {
                            ps.ok = false;
                            break;
                        }
                        t.begin = o[0];
                        t.end = o[1];
                    } else if (!ps.skip()) {
                        break;
                    }
                } while (ps.lit(','));
                if (ps.ok && !ps.lit('}')) ps.ok = false;
            }
            if (!ps.ok) break;
            if (t.begin < 0 || t.end < t.begin || data_start_ + t.end > file_size_) {
                err = "safetensors: tensor '" + t.name + "' has bad data_offsets";
                return G2_ERR_FORMAT;
            }
            tensors_.push_back(std::move(t));
        } while (ps.lit(','));
        if (ps.ok && !ps.lit('}')) ps.ok = false;
    }
    if (!ps.ok) {
        err = "safetensors: malformed header";
        return G2_ERR_FORMAT;
    }
    return G2_OK;
}

const StTensor *SafeTensors::find(const std::string &name) const {
    static const char *pre[3] = {"", "transformer.", "model."};
    for (const char *p : pre) {
        const std::string n = std::string(p) + name;
        for (const auto &t : tensors_)
            if (t.name == n) return &t;
    }
    return nullptr;
}

static float half_bits_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else {
            int sh = 0;
            while (!(m & 0x400)) {
                m <<= 1;
                ++sh;
            }
            u = s | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int SafeTensors::read_f32(const StTensor &t, float *out, std::string &err) {
    const int64_t n = t.numel();
    const int es = t.dtype == ST_F32 ? 4 : (t.dtype == ST_F16 || t.dtype == ST_BF16) ? 2 : 0;
    if (!es) {
        err = "tensor '" + t.name + "': unsupported dtype (F32, F16, BF16 accepted)";
        return G2_ERR_FORMAT;
    }
    if (t.end - t.begin != n * es) {
        err = "tensor '" + t.name + "': byte size does not match shape";
        return G2_ERR_FORMAT;
    }
    if (fseeko(fp_, data_start_ + t.begin, SEEK_SET) != 0) {
        err = "seek failed";
        return G2_ERR_IO;
    }
    if (es == 4) {
        if (fread(out, 4, (size_t)n, fp_) != (size_t)n) {
            err = "short read of '" + t.name + "'";
            return G2_ERR_IO;
        }
        return G2_OK;
    }
    std::vector<uint16_t> tmp((size_t)n);
    if (fread(tmp.data(), 2, (size_t)n, fp_) != (size_t)n) {
        err = "short read of '" + t.name + "'";
        return G2_ERR_IO;
    }
    for (int64_t i = 0; i < n; ++i) {
        if (t.dtype == ST_F16) {
            out[i] = half_bits_to_float(tmp[i]);
        } else {
            uint32_t u = (uint32_t)tmp[i] << 16;
            memcpy(&out[i], &u, 4);
        }
    }
    return G2_OK;
}

int validate_gpt2(const std::string &dir, const ModelConfig &c, std::string &err) {
    SafeTensors sf;
    int rc = sf.open(dir + "/model.safetensors", err);
    if (rc) return rc;
    const int64_t E = c.n_embd, F = c.ffn_dim, V = c.vocab_size;
    const StTensor *probe = sf.find("h.0.attn.c_attn.weight");
    if (!probe || probe->shape.size() != 2) {
        err = "cannot find h.0.attn.c_attn.weight";
        return G2_ERR_FORMAT;
    }
    bool conv1d;
    if (probe->shape[0] == E && probe->shape[1] == 3 * E) conv1d = true;
    else if (probe->shape[0] == 3 * E && probe->shape[1] == E) conv1d = false;
    else {
        err = "h.0.attn.c_attn.weight: unexpected shape";
        return G2_ERR_FORMAT;
    }
    struct Need {
        std::string name;
        int64_t rows, cols;   // cols == 0: vector of `rows`
        bool linear;
    };
    std::vector<Need> need = {{"wte.weight", V, E, false}, {"wpe.weight", c.n_ctx, E, false},
                              {"ln_f.weight", E, 0, false}, {"ln_f.bias", E, 0, false}};
    for (int l = 0; l < c.n_layer; ++l) {
        const std::string p = "h." + std::to_string(l) + ".";
        need.push_back({p + "ln_1.weight", E, 0, false});
        need.push_back({p + "ln_1.bias", E, 0, false});
        need.push_back({p + "attn.c_attn.weight", E, 3 * E, true});
        need.push_back({p + "attn.c_attn.bias", 3 * E, 0, false});
        need.push_back({p + "attn.c_proj.weight", E, E, true});
        need.push_back({p + "attn.c_proj.bias", E, 0, false});
        need.push_back({p + "ln_2.weight", E, 0, false});
        need.push_back({p + "ln_2.bias", E, 0, false});
        need.push_back({p + "mlp.c_fc.weight", E, F, true});
        need.push_back({p + "mlp.c_fc.bias", F, 0, false});
        need.push_back({p + "mlp.c_proj.weight", F, E, true});
        need.push_back({p + "mlp.c_proj.bias", E, 0, false});
    }
    for (const auto &n : need) {
        const StTensor *t = sf.find(n.name);
        if (!t) {
            err = "tensor '" + n.name + "' not found";
            return G2_ERR_FORMAT;
        }
        if (t->dtype == ST_OTHER) {
            err = "tensor '" + n.name + "': unsupported dtype (F32, F16, BF16 accepted)";
            return G2_ERR_FORMAT;
        }
        const int64_t want = n.cols ? n.rows * n.cols : n.rows;
        bool shape_ok = t->numel() == want;
        if (shape_ok && n.cols) {
            shape_ok = t->shape.size() == 2;
            if (shape_ok && n.linear && !conv1d) shape_ok = t->shape[0] == n.cols && t->shape[1] == n.rows;
            else if (shape_ok) shape_ok = t->shape[0] == n.rows && t->shape[1] == n.cols;
        }
        if (!shape_ok) {
            err = "tensor '" + n.name + "': shape does not match config";
            return G2_ERR_FORMAT;
        }
        const int es = t->dtype == ST_F32 ? 4 : 2;
        if (t->end - t->begin != t->numel() * es) {
            err = "tensor '" + n.name + "': byte size does not match shape";
            return G2_ERR_FORMAT;
        }
    }
    if (const StTensor *lm = sf.find("lm_head.weight")) {
        if (lm->shape.size() != 2 || !((lm->shape[0] == V && lm->shape[1] == E) || (lm->shape[0] == E && lm->shape[1] == V))) {
            err = "lm_head.weight: unexpected shape";
            return G2_ERR_FORMAT;
        }
    }
    return G2_OK;
}

}  // namespace g2
