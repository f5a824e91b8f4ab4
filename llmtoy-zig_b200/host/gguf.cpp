// gguf.cpp — GGUF parsing, the info report and the model loader (gguf.h).
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

namespace {

constexpr uint32_t kMagic = 0x46554747;  // "GGUF", src/gguf/types.zig:3
constexpr uint64_t kAlign = 32;          // types.zig:4

enum MetaType : uint32_t { U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };

struct Meta {
    uint32_t type = 0;
    uint64_t u = 0;  // unsigned / bool / bit pattern of signed
    double f = 0.0;
    std::string s;
    uint64_t count = 0;  // arrays: element count
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;  // innermost first
    uint32_t type = 0;
    uint64_t offset = 0;
};

// Block geometry of the GGUF types (types.zig:138-173): elements, bytes.
bool block_of(uint32_t t, uint64_t &elems, uint64_t &bytes) {
    switch (t) {
    case 0: elems = 1; bytes = 4; return true;      // f32
    case 1: elems = 1; bytes = 2; return true;      // f16
    case 2: elems = 32; bytes = 18; return true;    // q4_0
    case 3: elems = 32; bytes = 20; return true;    // q4_1
    case 6: elems = 32; bytes = 22; return true;    // q5_0
    case 7: elems = 32; bytes = 24; return true;    // q5_1
    case 8: elems = 32; bytes = 34; return true;    // q8_0
    case 10: elems = 256; bytes = 84; return true;  // q2_k
    case 11: elems = 256; bytes = 110; return true; // q3_k
    case 12: elems = 256; bytes = 144; return true; // q4_k
    case 13: elems = 256; bytes = 176; return true; // q5_k
    case 14: elems = 256; bytes = 210; return true; // q6_k
    case 20: elems = 32; bytes = 18; return true;   // iq4_nl
    case 30: elems = 1; bytes = 2; return true;     // bf16
    default: return false;
    }
}

const char *type_label(uint32_t t) {
    switch (t) {
    case 0: return "f32";
    case 1: return "f16";
    case 2: return "q4_0";
    case 3: return "q4_1";
    case 6: return "q5_0";
    case 7: return "q5_1";
    case 8: return "q8_0";
    case 10: return "q2_k";
    case 11: return "q3_k";
    case 12: return "q4_k";
    case 13: return "q5_k";
    case 14: return "q6_k";
    case 20: return "iq4_nl";
    case 30: return "bf16";
    default: return "other";
    }
}

// The types this backend decodes on the device (lt_upload accepts).
bool device_type(uint32_t t) {
    return t == 0 || t == 1 || t == 6 || t == 7 || t == 8 || t == 11 || t == 12 || t == 13 || t == 14 || t == 20;
}

struct Cursor {
    const uint8_t *p;
    size_t n, pos = 0;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if (pos + sizeof(T) > n) {
            ok = false;
            return v;
        }
        std::memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > n - pos) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(p + pos), len);
        pos += len;
        return s;
    }
};

bool read_value(Cursor &c, uint32_t t, Meta &m, int depth) {
    m.type = t;
    switch (t) {
    case U8: m.u = c.get<uint8_t>(); break;
    case I8: m.u = (uint64_t)(int64_t)c.get<int8_t>(); break;
    case U16: m.u = c.get<uint16_t>(); break;
    case I16: m.u = (uint64_t)(int64_t)c.get<int16_t>(); break;
    case U32: m.u = c.get<uint32_t>(); break;
    case I32: m.u = (uint64_t)(int64_t)c.get<int32_t>(); break;
    case F32: m.f = c.get<float>(); break;
    case BOOL: m.u = c.get<uint8_t>() != 0; break;
    case STR: m.s = c.str(); break;
    case U64: m.u = c.get<uint64_t>(); break;
    case I64: m.u = (uint64_t)c.get<int64_t>(); break;
    case F64: m.f = c.get<double>(); break;
    case ARR: {
        if (depth > 4) return false;
        const uint32_t et = c.get<uint32_t>();
        m.count = c.get<uint64_t>();
        for (uint64_t i = 0; i < m.count && c.ok; i++) {
            Meta e;
            if (!read_value(c, et, e, depth + 1)) return false;
        }
        break;
    }
    default: return false;
    }
    return c.ok;
}

}  // namespace

struct lth_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    std::map<std::string, Meta> meta;
    std::vector<TensorInfo> tensors;
    std::map<std::string, size_t> by_name;
    uint64_t data_offset = 0;

    bool meta_u64(const std::string &k, uint64_t &v) const {
        auto it = meta.find(k);
        if (it == meta.end() || (it->second.type != U32 && it->second.type != U64)) return false;
        v = it->second.u;
        return true;
    }
    bool meta_u32(const std::string &k, uint64_t &v) const {
        auto it = meta.find(k);
        if (it == meta.end() || it->second.type != U32) return false;
        v = it->second.u;
        return true;
    }
    bool meta_f32(const std::string &k, float &v) const {
        auto it = meta.find(k);
        if (it == meta.end() || it->second.type != F32) return false;
        v = (float)it->second.f;
        return true;
    }
    const std::string *meta_str(const std::string &k) const {
        auto it = meta.find(k);
        return it == meta.end() || it->second.type != STR ? nullptr : &it->second.s;
    }
    const TensorInfo *tensor(const std::string &name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : &tensors[it->second];
    }
    uint64_t nbytes(const TensorInfo &t) const {
        uint64_t e = 0, b = 0;
        if (!block_of(t.type, e, b) || t.dims.empty()) return 0;
        uint64_t n = (t.dims[0] / e) * b;
        for (size_t i = 1; i < t.dims.size(); i++) n *= t.dims[i];
        return n;
    }
    const uint8_t *bytes(const TensorInfo &t) const { return map + data_offset + t.offset; }
};

extern "C" {

lt_status lth_gguf_open(const char *path, lth_gguf **out) {
    if (!path || !out) return LT_EINVAL;
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return LT_EINVAL;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size == 0) {
        close(fd);
        return LT_EINVAL;
    }
    void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        close(fd);
        return LT_ENOMEM;
    }
    lth_gguf *g = new (std::nothrow) lth_gguf;
    if (!g) {
        munmap(m, (size_t)st.st_size);
        close(fd);
        return LT_ENOMEM;
    }
    g->fd = fd;
    g->map = static_cast<const uint8_t *>(m);
    g->size = (size_t)st.st_size;
    Cursor c{g->map, g->size};
    bool ok = c.get<uint32_t>() == kMagic;
    g->version = c.get<uint32_t>();
    ok = ok && c.ok && g->version >= 1 && g->version <= 3;
    // v1 counts are u32, v2+ u64 (reader.zig:70-72)
    const uint64_t n_tensors = !ok ? 0 : g->version == 1 ? c.get<uint32_t>() : c.get<uint64_t>();
    const uint64_t n_kv = !ok ? 0 : g->version == 1 ? c.get<uint32_t>() : c.get<uint64_t>();
    ok = ok && c.ok && n_tensors < (1u << 24) && n_kv < (1u << 24);
    for (uint64_t i = 0; ok && i < n_kv; i++) {
        std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        Meta v;
        ok = c.ok && read_value(c, t, v, 0);
        if (ok) g->meta[key] = std::move(v);
    }
    for (uint64_t i = 0; ok && i < n_tensors; i++) {
        TensorInfo ti;
        ti.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        ok = c.ok && nd >= 1 && nd <= 4;
        for (uint32_t j = 0; ok && j < nd; j++) ti.dims.push_back(c.get<uint64_t>());
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        ok = ok && c.ok;
        if (ok) {
            g->by_name[ti.name] = g->tensors.size();
            g->tensors.push_back(std::move(ti));
        }
    }
    if (ok) {
        g->data_offset = (c.pos + kAlign - 1) / kAlign * kAlign;
        for (const TensorInfo &t : g->tensors) {  // every tensor must lie inside the file
            const uint64_t nb = g->nbytes(t);
            if (nb != 0 && (g->data_offset + t.offset > g->size || nb > g->size - g->data_offset - t.offset)) ok = false;
        }
    }
    if (!ok) {
        lth_gguf_close(g);
        return LT_EINVAL;
    }
    *out = g;
    return LT_OK;
}

void lth_gguf_close(lth_gguf *g) {
    if (!g) return;
    if (g->map) munmap(const_cast<uint8_t *>(g->map), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

uint64_t lth_gguf_tensor_count(const lth_gguf *g) { return g ? g->tensors.size() : 0; }

lt_status lth_gguf_tensor(const lth_gguf *g, uint64_t i, const char **name, uint32_t *ggml_type, uint64_t *nbytes) {
    if (!g || i >= g->tensors.size()) return LT_EINVAL;
    const TensorInfo &t = g->tensors[i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (nbytes) *nbytes = g->nbytes(t);
    return LT_OK;
}

size_t lth_gguf_info(const lth_gguf *g, char *buf, size_t size) {
    if (!g) return 0;
    std::string o;
    char line[512];
    auto put = [&](const char *fmt, auto... a) {
        snprintf(line, sizeof line, fmt, a...);
        o += line;
    };
    auto dims = [](const TensorInfo &t) {
        std::string s = "{ ";
        for (size_t i = 0; i < t.dims.size(); i++) s += (i ? ", " : "") + std::to_string(t.dims[i]);
        return s + " }";
    };
    put("version:   GGUF v%u\n", g->version);
    put("size:      %.2f GiB\n", (double)g->size / (1024.0 * 1024.0 * 1024.0));
    put("tensors:   %zu\n", g->tensors.size());
    put("metadata:  %zu entries\n", g->meta.size());
    if (const std::string *arch = g->meta_str("general.architecture")) {
        put("arch:      %s\n", arch->c_str());
        uint64_t v;
        if (g->meta_u32(*arch + ".context_length", v)) put("ctx_len:   %llu\n", (unsigned long long)v);
        if (g->meta_u32(*arch + ".embedding_length", v)) put("emb_dim:   %llu\n", (unsigned long long)v);
        if (g->meta_u32(*arch + ".block_count", v)) put("n_layers:  %llu\n", (unsigned long long)v);
        if (g->meta_u32(*arch + ".attention.head_count", v)) put("n_heads:   %llu\n", (unsigned long long)v);
    }
    if (const std::string *n = g->meta_str("general.name")) put("name:      %s\n", n->c_str());
    if (const std::string *t = g->meta_str("tokenizer.chat_template")) {
        const size_t e = t->find('\n');
        put("chat_tmpl: present (%zu bytes), first line: %s\n", t->size(), t->substr(0, e).c_str());
    }
    uint64_t v;
    if (g->meta_u64("gemma4.embedding_length_per_layer_input", v)) put("per_layer_input: %llu\n", (unsigned long long)v);
    if (g->meta_u64("gemma4.attention.shared_kv_layers", v)) put("shared_kv_layers: %llu\n", (unsigned long long)v);
    if (g->meta_u32("tokenizer.ggml.bos_token_id", v)) put("bos_token: %llu\n", (unsigned long long)v);
    if (g->meta_u32("tokenizer.ggml.eos_token_id", v)) put("eos_token: %llu\n", (unsigned long long)v);
    o += "\nquant distribution:\n";
    std::map<uint32_t, uint32_t> counts;
    for (const TensorInfo &t : g->tensors) counts[t.type]++;
    for (auto &kv : counts) put("  %s: %u\n", type_label(kv.first), kv.second);
    // the reference lists the tensors its GPU backend cannot decode; here:
    // the types this backend's device kernels decode (F32, F16, Q5_0, Q5_1, Q8_0, Q3_K, Q4_K, Q5_K,
    // Q6_K, IQ4_NL)
    o += "\nunsupported GPU quant tensors:\n";
    size_t bad = 0;
    for (const TensorInfo &t : g->tensors) {
        if (device_type(t.type)) continue;
        bad++;
        put("  [%s] %s  dims=%s\n", type_label(t.type), t.name.c_str(), dims(t).c_str());
    }
    if (!bad) o += "  none\n";
    o += "\nfirst 16 tensors:\n";
    for (size_t i = 0; i < g->tensors.size() && i < 16; i++)
        put("  [%s] %s  dims=%s\n", type_label(g->tensors[i].type), g->tensors[i].name.c_str(),
            dims(g->tensors[i]).c_str());
    for (const char *prefix : {"blk.0.", "blk.5."}) {
        put("\n%s* tensors:\n", prefix);
        for (const TensorInfo &t : g->tensors)
            if (t.name.rfind(prefix, 0) == 0)
                put("  [%s] %s  dims=%s\n", type_label(t.type), t.name.c_str(), dims(t).c_str());
    }
    if (buf && size) {
        const size_t n = o.size() < size - 1 ? o.size() : size - 1;
        std::memcpy(buf, o.data(), n);
        buf[n] = 0;
    }
    return o.size();
}

}  // extern "C"

// ── model loader ───────────────────────────────────────────────────────────

struct lth_loaded {
    lt_ctx *ctx = nullptr;
    std::vector<lt_tensor *> tensors;
    std::vector<void *> bufs;
    std::vector<lth_layer> layers;
    lth_model model{};
    lth_decoder *dec = nullptr;
    uint32_t shape[8] = {};
};

namespace {

float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {  // subnormal
            int ee = -1;
            uint32_t mm = m;
            do {
                ee++;
                mm <<= 1;
            } while (!(mm & 1024));
            bits = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

struct Loader {
    lt_ctx *ctx;
    const lth_gguf *g;
    lth_loaded *out;
    std::string err;

    const TensorInfo *need(const std::string &name) {
        const TensorInfo *t = g->tensor(name);
        if (!t) err = "missing tensor " + name;
        return t;
    }
    // loadNorm / loadBias (loader.zig:152-188): f32 or f16 vectors of n values -> device f32
    lt_status vec(const TensorInfo *t, uint64_t n, const float **dev) {
        if (!t || t->dims.empty() || t->dims[0] != n || (t->type != 0 && t->type != 1)) {
            err = "bad vector tensor";
            return LT_EINVAL;
        }
        std::vector<float> h(n);
        const uint8_t *b = g->bytes(*t);
        for (uint64_t i = 0; i < n; i++) {
            if (t->type == 0) {
                std::memcpy(&h[i], b + 4 * i, 4);
            } else {
                uint16_t x;
                std::memcpy(&x, b + 2 * i, 2);
                h[i] = f16_to_f32(x);
            }
        }
        void *d = nullptr;
        lt_status st = lt_device_alloc(ctx, n * 4, &d);
        if (st != LT_OK) return st;
        out->bufs.push_back(d);
        if ((st = lt_copy_to_device(ctx, d, h.data(), n * 4)) != LT_OK) return st;
        if ((st = lt_sync(ctx)) != LT_OK) return st;
        *dev = static_cast<const float *>(d);
        return LT_OK;
    }
    // rawMatrix (loader.zig:190-203) uploaded: rows x cols (per expert when n_experts)
    lt_status mat(const TensorInfo *t, uint64_t rows, uint64_t cols, uint32_t n_experts, const lt_tensor **res) {
        if (!t) return LT_EINVAL;
        const uint64_t want_dims = n_experts ? 3 : 2;
        if (t->dims.size() < want_dims || t->dims[0] != cols || t->dims[1] != rows ||
            (n_experts && t->dims[2] != n_experts)) {
            err = "unexpected shape of " + t->name;
            return LT_EINVAL;
        }
        lt_tensor *h = nullptr;
        lt_status st = lt_upload(ctx, g->bytes(*t), g->nbytes(*t), t->type, rows, cols, n_experts, &h);
        if (st != LT_OK) {
            err = "upload of " + t->name + ": " + lt_last_error(ctx);
            return st;
        }
        out->tensors.push_back(h);
        *res = h;
        return LT_OK;
    }
    // Q, K and V rows stacked into one tensor (one matvec) when their types agree
    lt_status qkv(const TensorInfo *q, const TensorInfo *k, const TensorInfo *v, uint64_t nq, uint64_t nkv, uint64_t d,
                  lth_layer &L) {
        if (q->type == k->type && q->type == v->type && q->dims.size() == 2 && k->dims.size() == 2 &&
            v->dims.size() == 2 && q->dims[0] == d && k->dims[0] == d && v->dims[0] == d && q->dims[1] == nq &&
            k->dims[1] == nkv && v->dims[1] == nkv) {
            std::vector<uint8_t> buf;
            for (const TensorInfo *t : {q, k, v}) buf.insert(buf.end(), g->bytes(*t), g->bytes(*t) + g->nbytes(*t));
            lt_tensor *h = nullptr;
            lt_status st = lt_upload(ctx, buf.data(), buf.size(), q->type, nq + 2 * nkv, d, 0, &h);
            if (st != LT_OK) return st;
            out->tensors.push_back(h);
            L.wqkv = h;
            return LT_OK;
        }
        lt_status st;
        if ((st = mat(q, nq, d, 0, &L.wq)) != LT_OK) return st;
        if ((st = mat(k, nkv, d, 0, &L.wk)) != LT_OK) return st;
        return mat(v, nkv, d, 0, &L.wv);
    }
};

}  // namespace

extern "C" {

lt_status lth_model_load(lt_ctx *ctx, const lth_gguf *g, uint32_t kv_cap, lth_loaded **out) {
    if (!ctx || !g || !out || kv_cap == 0) return LT_EINVAL;
    *out = nullptr;
    const std::string *archp = g->meta_str("general.architecture");
    if (!archp) return LT_EINVAL;
    const std::string arch = *archp;
    uint64_t d = 0, L = 0, nh = 0, nkvh = 0, ff = 0, vocab = 0, hd = 0, E = 0, k = 0, fe = 0;
    // configFromGguf (loader.zig:37-83)
    if (!g->meta_u64(arch + ".embedding_length", d) || !g->meta_u64(arch + ".block_count", L) ||
        !g->meta_u64(arch + ".attention.head_count", nh) || !g->meta_u64(arch + ".attention.head_count_kv", nkvh))
        return LT_EINVAL;
    g->meta_u64(arch + ".feed_forward_length", ff);
    if (!g->meta_u64(arch + ".vocab_size", vocab) && !g->meta_u64("tokenizer.ggml.vocab_size", vocab)) {
        auto it = g->meta.find("tokenizer.ggml.tokens");
        if (it == g->meta.end() || it->second.type != ARR) {
            const TensorInfo *emb = g->tensor("token_embd.weight");
            if (!emb || emb->dims.size() != 2) return LT_EINVAL;
            vocab = emb->dims[1];
        } else {
            vocab = it->second.count;
        }
    }
    float eps = 1e-5f, theta = 500000.0f;
    g->meta_f32(arch + ".attention.layer_norm_rms_epsilon", eps);
    g->meta_f32(arch + ".rope.freq_base", theta);
    if (!g->meta_u64(arch + ".attention.key_length", hd)) hd = nh ? d / nh : 0;
    const bool moe = g->meta_u64(arch + ".expert_count", E) && E > 0;
    if (moe) {
        g->meta_u64(arch + ".expert_used_count", k);
        if (!g->meta_u64(arch + ".expert_feed_forward_length", fe)) fe = ff;
    }
    if (!d || !L || !nh || !nkvh || !hd || !vocab || nh % nkvh || (moe && (!k || !fe))) return LT_EINVAL;

    lth_loaded *m = new (std::nothrow) lth_loaded;
    if (!m) return LT_ENOMEM;
    m->ctx = ctx;
    Loader ld{ctx, g, m, {}};
    lt_status st = LT_OK;
    const uint64_t nq = nh * hd, nkv = nkvh * hd;
    m->layers.resize(L);
    auto name = [](uint64_t l, const char *s) { return "blk." + std::to_string(l) + "." + s; };
    for (uint64_t l = 0; l < L && st == LT_OK; l++) {
        lth_layer &ly = m->layers[l];
        std::memset(&ly, 0, sizeof ly);
        const TensorInfo *q = ld.need(name(l, "attn_q.weight")), *kk = ld.need(name(l, "attn_k.weight"));
        const TensorInfo *v = ld.need(name(l, "attn_v.weight")), *o = ld.need(name(l, "attn_output.weight"));
        if (!q || !kk || !v || !o) {
            st = LT_EINVAL;
            break;
        }
        if ((st = ld.vec(ld.need(name(l, "attn_norm.weight")), d, &ly.attn_norm)) != LT_OK) break;
        if ((st = ld.vec(ld.need(name(l, "ffn_norm.weight")), d, &ly.ffn_norm)) != LT_OK) break;
        if ((st = ld.qkv(q, kk, v, nq, nkv, d, ly)) != LT_OK) break;
        if ((st = ld.mat(o, d, nq, 0, &ly.wo)) != LT_OK) break;
        // optional Q/K/V biases (loader.zig:128-131), stacked like the rows
        const TensorInfo *qb = g->tensor(name(l, "attn_q.bias")), *kb = g->tensor(name(l, "attn_k.bias"));
        const TensorInfo *vb = g->tensor(name(l, "attn_v.bias"));
        if (qb && kb && vb) {
            std::vector<float> b;
            for (const TensorInfo *t : {qb, kb, vb}) {
                if (t->type != 0) {
                    st = LT_EINVAL;
                    break;
                }
                const float *p = reinterpret_cast<const float *>(g->bytes(*t));
                b.insert(b.end(), p, p + t->dims[0]);
            }
            if (st != LT_OK || b.size() != nq + 2 * nkv) {
                st = LT_EINVAL;
                break;
            }
            void *dv = nullptr;
            if ((st = lt_device_alloc(ctx, b.size() * 4, &dv)) != LT_OK) break;
            m->bufs.push_back(dv);
            if ((st = lt_copy_to_device(ctx, dv, b.data(), b.size() * 4)) != LT_OK || (st = lt_sync(ctx)) != LT_OK)
                break;
            ly.qkv_bias = static_cast<const float *>(dv);
        }
        const TensorInfo *qn = g->tensor(name(l, "attn_q_norm.weight")), *kn = g->tensor(name(l, "attn_k_norm.weight"));
        if (qn && (st = ld.vec(qn, hd, &ly.q_norm)) != LT_OK) break;
        if (kn && (st = ld.vec(kn, hd, &ly.k_norm)) != LT_OK) break;
        if (moe) {
            if ((st = ld.mat(ld.need(name(l, "ffn_gate_inp.weight")), E, d, 0, &ly.router)) != LT_OK) break;
            if ((st = ld.mat(ld.need(name(l, "ffn_gate_exps.weight")), fe, d, (uint32_t)E, &ly.exp_gate)) != LT_OK) break;
            if ((st = ld.mat(ld.need(name(l, "ffn_up_exps.weight")), fe, d, (uint32_t)E, &ly.exp_up)) != LT_OK) break;
            if ((st = ld.mat(ld.need(name(l, "ffn_down_exps.weight")), d, fe, (uint32_t)E, &ly.exp_down)) != LT_OK) break;
        } else {
            if ((st = ld.mat(ld.need(name(l, "ffn_gate.weight")), ff, d, 0, &ly.ffn_gate)) != LT_OK) break;
            if ((st = ld.mat(ld.need(name(l, "ffn_up.weight")), ff, d, 0, &ly.ffn_up)) != LT_OK) break;
            if ((st = ld.mat(ld.need(name(l, "ffn_down.weight")), d, ff, 0, &ly.ffn_down)) != LT_OK) break;
        }
    }
    lth_model &md = m->model;
    if (st == LT_OK) {
        const TensorInfo *emb = ld.need("token_embd.weight");
        st = ld.mat(emb, vocab, d, 0, &md.token_emb);
        // the LM head falls back to the embedding when absent (loader.zig:112-113)
        const TensorInfo *outw = g->tensor("output.weight");
        if (st == LT_OK) st = outw ? ld.mat(outw, vocab, d, 0, &md.lm_head) : (md.lm_head = md.token_emb, LT_OK);
        if (st == LT_OK) st = ld.vec(ld.need("output_norm.weight"), d, &md.out_norm);
    }
    if (st == LT_OK) {
        md.n_layers = (uint32_t)L;
        md.d_model = (uint32_t)d;
        md.n_heads = (uint32_t)nh;
        md.n_kv_heads = (uint32_t)nkvh;
        md.head_dim = (uint32_t)hd;
        md.vocab = (uint32_t)vocab;
        md.n_used = (uint32_t)k;
        // Qwen3-MoE renormalises the selected weights and rotates NeoX halves;
        // the dense llama-style loop rotates consecutive pairs (forward.zig:289-290)
        md.norm_topk = moe ? 1u : 0u;
        md.rope_neox = (arch == "qwen3moe" || arch == "qwen3") ? 1u : 0u;
        md.act = LT_ACT_SILU;
        md.eps = eps;
        md.rope_theta = theta;
        md.kv_cap = kv_cap;
        md.layers = m->layers.data();
        st = lth_decoder_create(ctx, &md, &m->dec);
    }
    if (st != LT_OK) {
        lth_loaded_free(m);
        return st;
    }
    const uint32_t sh[8] = {(uint32_t)L, (uint32_t)d, (uint32_t)nh, (uint32_t)nkvh, (uint32_t)hd, (uint32_t)vocab,
                            (uint32_t)E, (uint32_t)k};
    std::memcpy(m->shape, sh, sizeof sh);
    *out = m;
    return LT_OK;
}

lth_decoder *lth_loaded_decoder(const lth_loaded *m) { return m ? m->dec : nullptr; }

void lth_loaded_shape(const lth_loaded *m, uint32_t out[8]) {
    if (m && out) std::memcpy(out, m->shape, sizeof m->shape);
}

void lth_loaded_free(lth_loaded *m) {
    if (!m) return;
    if (m->dec) lth_decoder_free(m->dec);
    for (lt_tensor *t : m->tensors) lt_tensor_free(m->ctx, t);
    for (void *b : m->bufs) lt_device_free(m->ctx, b);
    delete m;
}

}  // extern "C"
