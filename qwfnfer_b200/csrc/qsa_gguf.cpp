// qsa_gguf.cpp -- QSA layer descriptors from a GGUF file's metadata (host code, C ABI).
//
// Reference: model_index::read_metadata (src/qwfn_model.cpp:111-152) reads the node's
// hyper-parameters under "<arch>." with typed getters and defaults (get_u32 accepts any integer
// type, get_f32 only F32, get_arr_i32 arrays of 32/64-bit integers; src/qwfn_model.cpp:17-95);
// hparams::is_attn_layer ((il + 1) % full_attention_interval == 0) and engine::init
// (src/qwfn_engine.cpp:384-431) make an attention layer with compress_ratios[il] > 0 a
// sparse-attention layer whose k_blocks = ceil((idx_top_k + r - 1) / r) includes the tail block.
//
// Only the metadata section is parsed (GGUF v2/v3: magic, version, tensor count, key/value count,
// then typed key/value pairs); tensor data is never touched.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qsa.h"

namespace {

enum GgufType : uint32_t {
    G_U8 = 0, G_I8 = 1, G_U16 = 2, G_I16 = 3, G_U32 = 4, G_I32 = 5, G_F32 = 6, G_BOOL = 7,
    G_STR = 8, G_ARR = 9, G_U64 = 10, G_I64 = 11, G_F64 = 12
};

struct Value {
    uint32_t type = 0;
    uint64_t u = 0;          // integer value (sign-extended into i when signed)
    int64_t  i = 0;
    float    f = 0.0f;
    std::string s;
    uint32_t arr_type = 0;
    std::vector<int64_t> arr_int;   // integer arrays only
    bool     arr_is_int = false;
};

struct Reader {
    FILE * f;
    bool ok = true;
    template <typename T> T get() {
        T v{};
        if (ok && std::fread(&v, sizeof v, 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 24)) { ok = false; return {}; }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
    void skip(uint64_t n) { if (ok && std::fseek(f, (long) n, SEEK_CUR) != 0) ok = false; }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case G_U8: case G_I8: case G_BOOL: return 1;
        case G_U16: case G_I16: return 2;
        case G_U32: case G_I32: case G_F32: return 4;
        case G_U64: case G_I64: case G_F64: return 8;
        default: return 0;
    }
}

bool read_int(Reader & r, uint32_t t, int64_t & out) {
    switch (t) {
        case G_U8:  out = r.get<uint8_t>(); return true;
        case G_I8:  out = r.get<int8_t>(); return true;
        case G_U16: out = r.get<uint16_t>(); return true;
        case G_I16: out = r.get<int16_t>(); return true;
        case G_U32: out = r.get<uint32_t>(); return true;
        case G_I32: out = r.get<int32_t>(); return true;
        case G_U64: out = (int64_t) r.get<uint64_t>(); return true;
        case G_I64: out = r.get<int64_t>(); return true;
        default: return false;
    }
}

bool read_value(Reader & r, uint32_t t, Value & v, bool keep) {
    v.type = t;
    if (t == G_STR) { v.s = r.str(); return r.ok; }
    if (t == G_F32) { v.f = r.get<float>(); return r.ok; }
    if (t == G_ARR) {
        v.arr_type = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (!r.ok) return false;
        const bool integer = v.arr_type == G_I32 || v.arr_type == G_U32 || v.arr_type == G_I64 || v.arr_type == G_U64;
        if (keep && integer && n <= 4096) {
            v.arr_is_int = true;
            v.arr_int.resize(n);
            for (uint64_t k = 0; k < n; k++) read_int(r, v.arr_type, v.arr_int[k]);
            return r.ok;
        }
        if (v.arr_type == G_STR) {
            for (uint64_t k = 0; k < n && r.ok; k++) r.str();
            return r.ok;
        }
        if (v.arr_type == G_ARR) return false;           // nested arrays: not metadata this reader needs
        const size_t es = scalar_size(v.arr_type);
        if (!es) return false;
        r.skip(n * es);
        return r.ok;
    }
    int64_t x = 0;
    if (read_int(r, t, x)) { v.i = x; v.u = (uint64_t) x; return r.ok; }
    if (t == G_BOOL) { v.u = r.get<uint8_t>(); return r.ok; }
    if (t == G_F64) { r.get<double>(); return r.ok; }
    return false;
}

struct Meta {
    std::vector<std::pair<std::string, Value>> kv;
    const Value * find(const std::string & k) const {
        for (const auto & p : kv) if (p.first == k) return &p.second;
        return nullptr;
    }
    // the reference loader's getters: any integer type for u32, F32 only for f32, integer arrays
    uint32_t u32(const std::string & k, uint32_t def) const {
        const Value * v = find(k);
        if (!v) return def;
        switch (v->type) {
            case G_U8: case G_I8: case G_U16: case G_I16: case G_U32: case G_I32: case G_U64: case G_I64:
                return (uint32_t) v->u;
            default: return def;
        }
    }
    float f32(const std::string & k, float def) const {
        const Value * v = find(k);
        return v && v->type == G_F32 ? v->f : def;
    }
    std::vector<int32_t> arr_i32(const std::string & k) const {
        const Value * v = find(k);
        std::vector<int32_t> out;
        if (!v || v->type != G_ARR || !v->arr_is_int) return out;
        for (int64_t x : v->arr_int) out.push_back((int32_t) x);
        return out;
    }
    std::string str(const std::string & k, const std::string & def) const {
        const Value * v = find(k);
        return v && v->type == G_STR ? v->s : def;
    }
};

void set_err(char * err, size_t n, const std::string & msg) {
    if (!err || !n) return;
    std::snprintf(err, n, "%s", msg.c_str());
}

bool read_meta(const char * path, Meta & m, std::string & err) {
    FILE * f = std::fopen(path, "rb");
    if (!f) { err = std::string("cannot open ") + path; return false; }
    Reader r{f};
    char magic[4];
    if (std::fread(magic, 1, 4, f) != 4 || std::memcmp(magic, "GGUF", 4) != 0) {
        std::fclose(f);
        err = "not a GGUF file";
        return false;
    }
    const uint32_t version = r.get<uint32_t>();
    if (!r.ok || version < 2 || version > 3) { std::fclose(f); err = "unsupported GGUF version"; return false; }
    r.get<uint64_t>();                                   // tensor count
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_kv > (1u << 20)) { std::fclose(f); err = "bad GGUF header"; return false; }
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        Value v;
        if (!r.ok || !read_value(r, t, v, true)) { r.ok = false; break; }
        m.kv.emplace_back(std::move(key), std::move(v));
    }
    std::fclose(f);
    if (!r.ok) { err = "truncated or malformed GGUF metadata"; return false; }
    return true;
}

}  // namespace

extern "C" qsa_status qsa_gguf_read_hparams(const char * path, qsa_gguf_hparams * hp, char * err, size_t err_len) {
    if (!path || !hp) return QSA_ERR_INVALID;
    Meta m;
    std::string e;
    if (!read_meta(path, m, e)) { set_err(err, err_len, e); return QSA_ERR_INVALID; }
    std::memset(hp, 0, sizeof *hp);
    const std::string arch = m.str("general.architecture", "");
    std::snprintf(hp->arch, sizeof hp->arch, "%s", arch.c_str());
    if (arch != "qwen4exp") {                            // model_index::read_metadata's check
        set_err(err, err_len, "unexpected architecture '" + arch + "'");
        return QSA_ERR_UNSUPPORTED;
    }
    const std::string A = arch + ".";
    hp->n_layer = (int32_t) m.u32(A + "block_count", 0);
    hp->n_embd = (int32_t) m.u32(A + "embedding_length", 0);
    hp->n_ctx_train = (int32_t) m.u32(A + "context_length", 0);
    hp->n_head = (int32_t) m.u32(A + "attention.head_count", 0);
    hp->n_head_kv = (int32_t) m.u32(A + "attention.head_count_kv", 0);
    hp->head_dim = (int32_t) m.u32(A + "attention.key_length", 0);
    hp->rms_eps = m.f32(A + "attention.layer_norm_rms_epsilon", 1e-6f);
    hp->full_attention_interval = (int32_t) m.u32(A + "full_attention_interval", 4);
    const std::vector<int32_t> cr = m.arr_i32(A + "attention.compress_ratios");
    if (cr.size() > QSA_GGUF_MAX_LAYERS) {
        set_err(err, err_len, "more layers than qsa_gguf_hparams holds");
        return QSA_ERR_UNSUPPORTED;
    }
    hp->n_compress = (int32_t) cr.size();
    for (size_t i = 0; i < cr.size(); i++) hp->compress_ratios[i] = cr[i];
    hp->rope_freq_base = m.f32(A + "rope.freq_base", 10000000.0f);
    hp->rope_dim = (int32_t) m.u32(A + "rope.dimension_count", 64);
    const std::vector<int32_t> secs = m.arr_i32(A + "rope.dimension_sections");
    const int32_t def_secs[4] = {11, 11, 10, 0};
    for (int i = 0; i < 4; i++) hp->sections[i] = i < (int) secs.size() ? secs[i] : def_secs[i];
    hp->idx_n_head = (int32_t) m.u32(A + "attention.indexer.head_count", 4);
    hp->idx_dim = (int32_t) m.u32(A + "attention.indexer.key_length", 128);
    hp->idx_top_k = (int32_t) m.u32(A + "attention.indexer.top_k", 2048);
    set_err(err, err_len, "");
    return QSA_OK;
}

extern "C" int32_t qsa_gguf_is_qsa_layer(const qsa_gguf_hparams * hp, int32_t il) {
    if (!hp || il < 0 || il >= hp->n_layer || hp->full_attention_interval <= 0) return 0;
    const bool attn = (il + 1) % hp->full_attention_interval == 0;          // hparams::is_attn_layer
    return attn && il < hp->n_compress && hp->compress_ratios[il] > 0 ? 1 : 0;
}

extern "C" qsa_status qsa_gguf_layer_desc(const qsa_gguf_hparams * hp, int32_t il, int32_t n_ctx, int32_t window,
                                          int32_t type_k, int32_t type_v, const float * k_norm_w, qsa_desc * out) {
    if (!hp || !out || n_ctx <= 0 || window < 0) return QSA_ERR_INVALID;
    if (!qsa_gguf_is_qsa_layer(hp, il)) return QSA_ERR_INVALID;
    const int32_t r = hp->compress_ratios[il];
    const int32_t k_blocks = (hp->idx_top_k + r - 1 + r - 1) / r;   // engine::init: ceil((top_k + r - 1) / r)
    qsa_desc d;
    std::memset(&d, 0, sizeof d);
    d.n_head = hp->n_head; d.n_head_kv = hp->n_head_kv; d.head_dim = hp->head_dim;
    d.idx_n_head = hp->idx_n_head; d.idx_dim = hp->idx_dim; d.ratio = r;
    d.top_k_blocks = k_blocks - 1;          // the reference forces its query's incomplete block: window 0
    d.window = window;
    d.n_ctx = (int32_t) (((int64_t) n_ctx + r - 1) / r * r);
    d.type_k = type_k; d.type_v = type_v;
    d.rope_dim = hp->rope_dim;
    for (int i = 0; i < 4; i++) d.sections[i] = hp->sections[i];
    d.rms_eps = hp->rms_eps; d.rope_freq_base = hp->rope_freq_base;
    d.k_norm_w = k_norm_w;
    *out = d;
    return qsa_desc_check(&d);
}
