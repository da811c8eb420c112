// GGUF checkpoint ingest: the model config from the file's metadata and every
// tensor of a llama / qwen3 GGUF into a model (fb_gguf_config,
// fb_model_load_gguf).
//
// Replaces what the reference does through candle's gguf_file::Content
// (crates/ferrite-wasm-host/src/adapter.rs:48-54, quantized_llama::
// ModelWeights::from_gguf) and its own metadata reader
// (crates/ferrite-core/src/registry/loader.rs:247-339, which keeps string and
// integer values only).  File layout (GGUF v2/v3, little endian): magic
// "GGUF", u32 version, u64 tensor count, u64 metadata count, the metadata
// (key string, u32 value type, value; arrays as u32 element type + u64 count
// + elements), the tensor infos (name, u32 n_dims, u64 dims innermost first,
// u32 ggml type, u64 offset into the data section), padding to
// general.alignment (default 32), the data section.
#include <stdio.h>
#include <string.h>
#include <sys/types.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "fb_internal.h"

namespace fb {
namespace {

enum GgufType : uint32_t {
    G_U8 = 0, G_I8, G_U16, G_I16, G_U32, G_I32, G_F32, G_BOOL, G_STRING, G_ARRAY, G_U64, G_I64, G_F64
};

struct Value {
    uint32_t type = 0;
    double num = 0.0;       // numeric scalars
    std::string str;        // strings
    uint64_t count = 0;     // arrays: element count
    uint32_t elem_type = 0;
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
};

struct File {
    FILE *f = nullptr;
    std::map<std::string, Value> kv;
    std::vector<TensorInfo> tensors;
    uint64_t data_offset = 0;
    ~File() {
        if (f) fclose(f);
    }
    void read(void *dst, size_t n) {
        if (fread(dst, 1, n, f) != n) fail(FB_ERR_INVALID, "gguf: unexpected end of file");
    }
    template <class T> T get() {
        T v;
        read(&v, sizeof(v));
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        FB_REQUIRE(n < (1ull << 30), "gguf: string length out of range");
        std::string s(n, '\0');
        if (n) read(&s[0], n);
        return s;
    }
    void skip_scalar(uint32_t t) {
        static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == G_STRING) {
            str();
            return;
        }
        FB_REQUIRE(t <= G_F64 && t != G_ARRAY, "gguf: bad value type");
        if (fseek(f, sz[t], SEEK_CUR) != 0) fail(FB_ERR_INVALID, "gguf: seek failed");
    }
    double num(uint32_t t) {
        switch (t) {
        case G_U8: return get<uint8_t>();
        case G_I8: return get<int8_t>();
        case G_U16: return get<uint16_t>();
        case G_I16: return get<int16_t>();
        case G_U32: return get<uint32_t>();
        case G_I32: return get<int32_t>();
        case G_F32: return get<float>();
        case G_BOOL: return get<uint8_t>();
        case G_U64: return (double)get<uint64_t>();
        case G_I64: return (double)get<int64_t>();
        case G_F64: return get<double>();
        default: fail(FB_ERR_INVALID, "gguf: not a numeric type");
        }
    }
};

std::unique_ptr<File> open_gguf(const char *path) {
    auto g = std::make_unique<File>();
    g->f = fopen(path, "rb");
    FB_REQUIRE(g->f, std::string("gguf: cannot open ") + path);
    char magic[4];
    g->read(magic, 4);
    FB_REQUIRE(memcmp(magic, "GGUF", 4) == 0, "gguf: bad magic");
    const uint32_t version = g->get<uint32_t>();
    FB_REQUIRE(version == 2 || version == 3, "gguf: only versions 2 and 3 are supported");
    const uint64_t n_tensors = g->get<uint64_t>(), n_kv = g->get<uint64_t>();
    FB_REQUIRE(n_tensors < (1u << 24) && n_kv < (1u << 24), "gguf: counts out of range");
    for (uint64_t i = 0; i < n_kv; i++) {
        const std::string key = g->str();
        Value v;
        v.type = g->get<uint32_t>();
        if (v.type == G_STRING) {
            v.str = g->str();
        } else if (v.type == G_ARRAY) {
            v.elem_type = g->get<uint32_t>();
            v.count = g->get<uint64_t>();
            FB_REQUIRE(v.elem_type != G_ARRAY, "gguf: nested arrays are not supported");
            for (uint64_t k = 0; k < v.count; k++) g->skip_scalar(v.elem_type);
        } else {
            v.num = g->num(v.type);
        }
        g->kv[key] = std::move(v);
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        TensorInfo t;
        t.name = g->str();
        const uint32_t nd = g->get<uint32_t>();
        FB_REQUIRE(nd >= 1 && nd <= 4, "gguf: tensor rank out of range");
        for (uint32_t d = 0; d < nd; d++) t.dims.push_back(g->get<uint64_t>());
        t.type = g->get<uint32_t>();
        t.offset = g->get<uint64_t>();
        g->tensors.push_back(std::move(t));
    }
    uint64_t align = 32;
    auto it = g->kv.find("general.alignment");
    if (it != g->kv.end() && it->second.type != G_STRING && it->second.type != G_ARRAY) align = (uint64_t)it->second.num;
    FB_REQUIRE(align >= 1 && align <= 65536, "gguf: bad alignment");
    const long pos = ftell(g->f);
    FB_REQUIRE(pos >= 0, "gguf: tell failed");
    g->data_offset = ((uint64_t)pos + align - 1) / align * align;
    return g;
}

double num_or(const File &g, const std::string &key, double dflt) {
    auto it = g.kv.find(key);
    if (it == g.kv.end() || it->second.type == G_STRING || it->second.type == G_ARRAY) return dflt;
    return it->second.num;
}
double num_req(const File &g, const std::string &key) {
    auto it = g.kv.find(key);
    FB_REQUIRE(it != g.kv.end() && it->second.type != G_STRING && it->second.type != G_ARRAY,
               "gguf: missing numeric metadata " + key);
    return it->second.num;
}
const TensorInfo *find_tensor(const File &g, const std::string &name) {
    for (const auto &t : g.tensors)
        if (t.name == name) return &t;
    return nullptr;
}

// ggml type id -> this library's dtype (k-quants and f32 share the numbering)
int dtype_of(uint32_t ggml_type) {
    switch (ggml_type) {
    case 0: return FB_F32;
    case 12: return FB_Q4_K;
    case 14: return FB_Q6_K;
    default: return -1;
    }
}
size_t tensor_bytes(const TensorInfo &t) {
    uint64_t n = 1;
    for (auto d : t.dims) n *= d;
    switch (t.type) {
    case 0: return (size_t)n * 4;
    case 12: return (size_t)(n / 256) * 144;
    case 14: return (size_t)(n / 256) * 210;
    default: return 0;
    }
}

void config_of(const File &g, fb_model_config &c, int &arch) {
    auto it = g.kv.find("general.architecture");
    FB_REQUIRE(it != g.kv.end() && it->second.type == G_STRING, "gguf: general.architecture missing");
    const std::string a = it->second.str;
    FB_REQUIRE(a == "llama" || a == "qwen3", "gguf: architecture '" + a + "' is not supported (llama, qwen3)");
    arch = a == "qwen3" ? 1 : 0;
    memset(&c, 0, sizeof(c));
    c.n_layers = (int)num_req(g, a + ".block_count");
    c.hidden = (int)num_req(g, a + ".embedding_length");
    c.ffn = (int)num_req(g, a + ".feed_forward_length");
    c.n_heads = (int)num_req(g, a + ".attention.head_count");
    c.n_kv_heads = (int)num_or(g, a + ".attention.head_count_kv", c.n_heads);
    c.head_dim = (int)num_or(g, a + ".attention.key_length", c.n_heads ? c.hidden / c.n_heads : 0);
    c.rope_theta = (float)num_or(g, a + ".rope.freq_base", 10000.0);
    c.eps = (float)num_or(g, a + ".attention.layer_norm_rms_epsilon", arch ? 1e-6 : 1e-5);
    c.max_ctx = (int)num_or(g, a + ".context_length", 4096);
    c.max_batch = 1;
    c.qk_norm = arch;    // qwen3: per-head RMSNorm of q and k
    c.rope_mode = arch;  // qwen3: rotate-half; llama GGUFs: interleaved pairs
    const TensorInfo *emb = find_tensor(g, "token_embd.weight");
    FB_REQUIRE(emb && emb->dims.size() == 2, "gguf: token_embd.weight missing");
    c.vocab = (int)emb->dims[1];
}

// GGUF tensor name -> (model tensor name, layer); false for tensors the
// model does not use (e.g. rope_freqs)
bool map_name(const std::string &n, std::string &out, int &layer) {
    const std::string suf = ".weight";
    if (n.size() <= suf.size() || n.compare(n.size() - suf.size(), suf.size(), suf) != 0) return false;
    std::string base = n.substr(0, n.size() - suf.size());
    layer = -1;
    if (base.rfind("blk.", 0) == 0) {
        const size_t dot = base.find('.', 4);
        if (dot == std::string::npos) return false;
        layer = std::stoi(base.substr(4, dot - 4));
        base = base.substr(dot + 1);
    }
    static const char *known[] = {"token_embd", "output_norm", "output",      "attn_norm",   "attn_q",
                                  "attn_k",     "attn_v",      "attn_output", "attn_q_norm", "attn_k_norm",
                                  "ffn_norm",   "ffn_gate",    "ffn_up",      "ffn_down"};
    for (const char *k : known)
        if (base == k) {
            out = base;
            return true;
        }
    return false;
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int fb_gguf_config(const char *path, fb_model_config *cfg_out, int *arch_out) {
    return guarded([&] {
        FB_REQUIRE(path && cfg_out, "null argument");
        auto g = open_gguf(path);
        int arch = 0;
        config_of(*g, *cfg_out, arch);
        if (arch_out) *arch_out = arch;
    });
}

int fb_model_load_gguf(fb_model *m, const char *path) {
    return guarded([&] {
        FB_REQUIRE(m && path, "null argument");
        auto g = open_gguf(path);
        std::vector<uint8_t> buf;
        bool have_output = false;
        for (const auto &t : g->tensors) {
            std::string name;
            int layer;
            if (!map_name(t.name, name, layer)) continue;
            const int dt = dtype_of(t.type);
            FB_REQUIRE(dt >= 0, "gguf: tensor " + t.name + " has ggml type " + std::to_string(t.type) +
                                    " (supported: F32, Q4_K, Q6_K)");
            const int64_t cols = (int64_t)t.dims[0], rows = t.dims.size() > 1 ? (int64_t)t.dims[1] : 1;
            const size_t bytes = tensor_bytes(t);
            buf.resize(bytes);
            if (fseeko(g->f, (off_t)(g->data_offset + t.offset), SEEK_SET) != 0)
                fail(FB_ERR_INVALID, "gguf: seek to tensor data failed");
            g->read(buf.data(), bytes);
            const int rc = fb_model_set_tensor(m, name.c_str(), layer, dt, rows, cols, buf.data());
            if (rc != FB_OK) fail(rc, fb_last_error());
            if (name == "output") have_output = true;
        }
        if (!have_output) {  // tied embeddings: the lm_head is token_embd
            const TensorInfo *e = find_tensor(*g, "token_embd.weight");
            FB_REQUIRE(e, "gguf: token_embd.weight missing");
            const int dt = dtype_of(e->type);
            FB_REQUIRE(dt == FB_Q4_K || dt == FB_Q6_K, "gguf: tied output needs a Q4_K / Q6_K token_embd");
            const size_t bytes = tensor_bytes(*e);
            buf.resize(bytes);
            if (fseeko(g->f, (off_t)(g->data_offset + e->offset), SEEK_SET) != 0)
                fail(FB_ERR_INVALID, "gguf: seek to tensor data failed");
            g->read(buf.data(), bytes);
            const int rc = fb_model_set_tensor(m, "output", -1, dt, (int64_t)e->dims[1], (int64_t)e->dims[0], buf.data());
            if (rc != FB_OK) fail(rc, fb_last_error());
        }
        const int rc = fb_model_finalize(m);
        if (rc != FB_OK) fail(rc, fb_last_error());
    });
}

}  // extern "C"
