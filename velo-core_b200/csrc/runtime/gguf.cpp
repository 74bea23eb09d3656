// gguf.cpp -- GGUF parsing, model metadata and validation on the host, and
// their C ABI (include/velo_cuda.h, velo_gguf_* and velo_cuda_load_gguf).
//
// Follows src/gguf.rs (GgufFile::read :227-287, read_value :392-421,
// read_array_elem :422-442, block_params :71-91) and src/model_loader.rs
// (ModelMeta::from_gguf :41-127, infer_quantization :143-153,
// WeightStore::validate :192-234, load_gguf :291-309).  Same acceptance rules
// and error kinds; the data section is memory-mapped instead of read into a
// buffer, so a 40 GB model costs no host copy before the device upload.
#include "runtime/gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "runtime/context.h"

namespace velo {

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint64_t kDefaultAlignment = 32;

struct Reader {
    const uint8_t* p;
    size_t n, pos = 0;
    bool take(void* dst, size_t k) {
        if (k > n - pos) return false;
        std::memcpy(dst, p + pos, k);
        pos += k;
        return true;
    }
    template <typename T>
    bool get(T* v) {
        return take(v, sizeof(T));
    }
};

int32_t eof() { return fail(VELO_ERR_IO, "I/O error: failed to fill whole buffer"); }

// Rust's String::from_utf8 acceptance: shortest forms only, no surrogates,
// nothing above U+10FFFF.
bool valid_utf8(const uint8_t* s, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int len;
        uint32_t cp;
        if ((c & 0xe0) == 0xc0) {
            len = 2;
            cp = c & 0x1f;
        } else if ((c & 0xf0) == 0xe0) {
            len = 3;
            cp = c & 0x0f;
        } else if ((c & 0xf8) == 0xf0) {
            len = 4;
            cp = c & 0x07;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (int j = 1; j < len; ++j) {
            if ((s[i + j] & 0xc0) != 0x80) return false;
            cp = (cp << 6) | (s[i + j] & 0x3f);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
            cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
            return false;
        i += len;
    }
    return true;
}

int32_t read_string(Reader& r, std::string* out) {
    uint64_t len = 0;
    if (!r.get(&len)) return eof();
    if (len > r.n - r.pos) return eof();
    const uint8_t* s = r.p + r.pos;
    if (!valid_utf8(s, (size_t)len)) return fail(VELO_ERR_GGUF, "malformed GGUF: invalid UTF-8 string");
    out->assign(reinterpret_cast<const char*>(s), (size_t)len);
    r.pos += (size_t)len;
    return VELO_OK;
}

// One value of type `t` (no tag); arrays only at the top level (`nested`
// false), as read_array_elem has no array case.
int32_t read_typed(Reader& r, uint32_t t, GgufValue* v, bool nested) {
    v->type = t;
    switch (t) {
    case 0: case 7: {
        uint8_t x;
        if (!r.get(&x)) return eof();
        v->u = t == 7 ? (x != 0) : x;
        return VELO_OK;
    }
    case 1: {
        int8_t x;
        if (!r.get(&x)) return eof();
        v->i = x;
        return VELO_OK;
    }
    case 2: {
        uint16_t x;
        if (!r.get(&x)) return eof();
        v->u = x;
        return VELO_OK;
    }
    case 3: {
        int16_t x;
        if (!r.get(&x)) return eof();
        v->i = x;
        return VELO_OK;
    }
    case 4: {
        uint32_t x;
        if (!r.get(&x)) return eof();
        v->u = x;
        return VELO_OK;
    }
    case 5: {
        int32_t x;
        if (!r.get(&x)) return eof();
        v->i = x;
        return VELO_OK;
    }
    case 6: {
        float x;
        if (!r.get(&x)) return eof();
        v->f = x;
        return VELO_OK;
    }
    case 8:
        return read_string(r, &v->s);
    case 9: {
        if (nested) break;
        uint32_t et;
        uint64_t count;
        if (!r.get(&et) || !r.get(&count)) return eof();
        v->u = et;  // element type of the array
        for (uint64_t k = 0; k < count; ++k) {
            GgufValue e;
            const int32_t st = read_typed(r, et, &e, true);
            if (st) return st;
            v->arr.push_back(std::move(e));
        }
        return VELO_OK;
    }
    case 10: {
        uint64_t x;
        if (!r.get(&x)) return eof();
        v->u = x;
        return VELO_OK;
    }
    case 11: {
        int64_t x;
        if (!r.get(&x)) return eof();
        v->i = x;
        return VELO_OK;
    }
    case 12: {
        double x;
        if (!r.get(&x)) return eof();
        v->f = x;
        return VELO_OK;
    }
    default:
        break;
    }
    return fail(VELO_ERR_GGUF, "unknown ggml type %u", t);
}

// GgufValue accessors (gguf.rs:120-193)
const GgufValue* find_meta(const GgufFile& g, const std::string& key) {
    auto it = g.meta.find(key);
    return it == g.meta.end() ? nullptr : &it->second;
}
bool as_u32(const GgufValue* v, uint64_t* out) {
    if (!v || v->type != 4) return false;
    *out = v->u;
    return true;
}
bool as_u64(const GgufValue* v, uint64_t* out) {
    if (!v || (v->type != 10 && v->type != 4)) return false;
    *out = v->u;
    return true;
}
bool as_f32(const GgufValue* v, float* out) {
    if (!v || v->type != 6) return false;
    *out = (float)v->f;
    return true;
}

std::string shape_str(const std::vector<uint64_t>& s) {
    std::string o = "[";
    for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
    return o + "]";
}

}  // namespace

bool ggml_block_params(uint32_t t, uint64_t* bytes, uint64_t* elems) {
    uint64_t b = 0, e = 1;
    switch (t) {
    case 0: case 26: b = 4; break;            // F32, I32
    case 1: case 25: case 30: b = 2; break;   // F16, I16, BF16
    case 2: b = 18; e = 32; break;            // Q4_0
    case 3: b = 20; e = 32; break;            // Q4_1
    case 6: b = 22; e = 32; break;            // Q5_0
    case 7: b = 24; e = 32; break;            // Q5_1
    case 8: b = 34; e = 32; break;            // Q8_0
    case 9: b = 36; e = 32; break;            // Q8_1
    case 10: b = 84; e = 256; break;          // Q2K
    case 11: b = 110; e = 256; break;         // Q3K
    case 12: b = 144; e = 256; break;         // Q4K
    case 13: b = 176; e = 256; break;         // Q5K
    case 14: b = 210; e = 256; break;         // Q6K
    case 15: b = 292; e = 256; break;         // Q8K
    case 24: b = 1; break;                    // I8
    case 27: case 28: b = 8; break;           // I64, F64
    default: return false;
    }
    *bytes = b;
    *elems = e;
    return true;
}

GgufFile::~GgufFile() {
    if (map_base) munmap(map_base, map_len);
}

int32_t gguf_read_header(const uint8_t* buf, size_t n, GgufFile& g, uint64_t* header_end) {
    Reader r{buf, n};
    uint32_t magic = 0, version = 0;
    if (!r.get(&magic)) return eof();
    if (magic != kMagic) return fail(VELO_ERR_GGUF, "bad magic: %#010x", magic);
    if (!r.get(&version)) return eof();
    if (version == 0 || version > 3) return fail(VELO_ERR_GGUF, "unsupported GGUF version %u", version);
    g.version = version;
    uint64_t n_tensors = 0, n_kv = 0;
    if (!r.get(&n_tensors) || !r.get(&n_kv)) return eof();
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        int32_t st = read_string(r, &key);
        if (st) return st;
        uint32_t t;
        if (!r.get(&t)) return eof();
        GgufValue v;
        st = read_typed(r, t, &v, false);
        if (st) return st;
        g.meta[key] = std::move(v);  // a repeated key keeps the last value
    }
    for (uint64_t k = 0; k < n_tensors; ++k) {
        GgufTensor ti;
        int32_t st = read_string(r, &ti.name);
        if (st) return st;
        uint32_t n_dims;
        if (!r.get(&n_dims)) return eof();
        if (n_dims > 4)
            return fail(VELO_ERR_GGUF, "malformed GGUF: tensor %s: too many dims (%u)", ti.name.c_str(), n_dims);
        ti.shape.resize(n_dims);
        for (auto& d : ti.shape)
            if (!r.get(&d)) return eof();
        if (!r.get(&ti.ggml_type)) return eof();
        uint64_t bb, be;
        if (!ggml_block_params(ti.ggml_type, &bb, &be)) return fail(VELO_ERR_GGUF, "unknown ggml type %u", ti.ggml_type);
        if (!r.get(&ti.offset)) return eof();
        // element count checked before every multiply, so no product can wrap
        unsigned __int128 ne = 1;
        bool too_large = false;
        for (uint64_t d : ti.shape) {
            if (d != 0 && ne > (unsigned __int128)UINT64_MAX / d) too_large = true;
            if (too_large) break;
            ne *= d;
        }
        const unsigned __int128 nb = too_large ? 0 : (ne + be - 1) / be * bb;
        if (too_large || ne >> 64 || nb >> 64)
            return fail(VELO_ERR_GGUF, "malformed GGUF: tensor %s is too large", ti.name.c_str());
        ti.nbytes = (uint64_t)nb;
        g.tensors[ti.name] = ti;  // a repeated name keeps the last entry
    }
    uint64_t align = kDefaultAlignment;
    const GgufValue* a = find_meta(g, "general.alignment");
    uint64_t av;
    if (as_u64(a, &av)) align = av;
    if (align == 0) return fail(VELO_ERR_GGUF, "malformed GGUF: general.alignment is 0");
    const uint64_t pos = r.pos;
    g.data_offset = (pos + align - 1) / align * align;
    if (header_end) *header_end = pos;
    return VELO_OK;
}

int32_t gguf_open(const char* path, GgufFile& g) {
    if (!path) return fail(VELO_ERR_INVALID_ARGUMENT, "path is NULL");
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return fail(VELO_ERR_IO, "I/O error loading %s: %s", path, std::strerror(errno));
    struct stat sb;
    if (fstat(fd, &sb) != 0) {
        const int e = errno;
        close(fd);
        return fail(VELO_ERR_IO, "I/O error loading %s: %s", path, std::strerror(e));
    }
    const size_t size = (size_t)sb.st_size;
    void* base = nullptr;
    if (size > 0) {
        base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (base == MAP_FAILED) {
            const int e = errno;
            close(fd);
            return fail(VELO_ERR_IO, "I/O error loading %s: %s", path, std::strerror(e));
        }
    }
    close(fd);  // the mapping stays valid
    g.map_base = base;
    g.map_len = size;
    const uint8_t* buf = static_cast<const uint8_t*>(base);
    int32_t st = gguf_read_header(buf, size, g, nullptr);
    if (st) return st;
    // read_all_tensors: the data section up to the furthest tensor end
    uint64_t end = 0;
    for (const auto& kv : g.tensors) {
        const uint64_t e = kv.second.offset + kv.second.nbytes;
        if (e < kv.second.offset) return fail(VELO_ERR_GGUF, "malformed GGUF: tensor %s offset overflows", kv.first.c_str());
        if (e > end) end = e;
    }
    if (end > 0 && (g.data_offset > size || end > size - g.data_offset)) return eof();
    g.data = end > 0 ? buf + g.data_offset : nullptr;
    g.data_bytes = end;
    return VELO_OK;
}

int32_t gguf_model_meta(const GgufFile& g, GgufModelMeta& m) {
    const GgufValue* a = find_meta(g, "general.architecture");
    m.arch = (a && a->type == 8) ? a->s : "llama";
    const std::string p = m.arch + ".";
    const GgufValue* toks = find_meta(g, "tokenizer.ggml.tokens");
    if (toks && toks->type == 9) {
        m.n_vocab = toks->arr.size();
    } else if (!as_u32(find_meta(g, p + "vocab_size"), &m.n_vocab)) {
        return fail(VELO_ERR_MISSING_META, "missing metadata key: vocab_size");
    }
    auto need = [&](const char* key, uint64_t* out) -> int32_t {
        if (as_u32(find_meta(g, p + key), out)) return VELO_OK;
        return fail(VELO_ERR_MISSING_META, "missing metadata key: %s%s", p.c_str(), key);
    };
    int32_t st = need("embedding_length", &m.n_embd);
    if (!st) st = need("block_count", &m.n_layer);
    if (!st) st = need("attention.head_count", &m.n_head);
    if (st) return st;
    if (!as_u32(find_meta(g, p + "attention.head_count_kv"), &m.n_head_kv)) m.n_head_kv = m.n_head;
    if (!as_u32(find_meta(g, p + "context_length"), &m.n_ctx)) m.n_ctx = 4096;
    st = need("feed_forward_length", &m.n_ff);
    if (st) return st;
    if (m.n_head == 0) return fail(VELO_ERR_GGUF, "malformed GGUF: %sattention.head_count is 0", p.c_str());
    m.head_dim = m.n_embd / m.n_head;
    if (!as_f32(find_meta(g, p + "rope.freq_base"), &m.rope_freq_base)) m.rope_freq_base = 10000.0f;
    if (!as_f32(find_meta(g, p + "attention.layer_norm_rms_epsilon"), &m.norm_eps)) m.norm_eps = 1e-5f;
    auto it = g.tensors.find("blk.0.attn_q.weight");
    if (it == g.tensors.end()) it = g.tensors.find("token_embd.weight");
    m.quantization = (it != g.tensors.end() && it->second.ggml_type == 12) ? 1 : 0;
    return VELO_OK;
}

int32_t gguf_validate(const GgufFile& g, const GgufModelMeta& m) {
    auto check = [&](const std::string& name, std::vector<uint64_t> want) -> int32_t {
        auto it = g.tensors.find(name);
        if (it == g.tensors.end()) return fail(VELO_ERR_MISSING_TENSOR, "missing tensor: %s", name.c_str());
        if (it->second.shape != want)
            return fail(VELO_ERR_INVALID_SHAPE, "tensor %s: expected shape %s, got %s", name.c_str(),
                        shape_str(want).c_str(), shape_str(it->second.shape).c_str());
        return VELO_OK;
    };
    const uint64_t E = m.n_embd, V = m.n_vocab, F = m.n_ff, KV = m.n_head_kv * m.head_dim;
    int32_t st = check("token_embd.weight", {E, V});
    for (uint64_t l = 0; !st && l < m.n_layer; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        st = check(p + "attention_norm.weight", {E});
        if (!st) st = check(p + "attention.wq.weight", {E, E});
        if (!st) st = check(p + "attention.wk.weight", {E, KV});
        if (!st) st = check(p + "attention.wv.weight", {E, KV});
        if (!st) st = check(p + "attention.wo.weight", {E, E});
        if (!st) st = check(p + "ffn_norm.weight", {E});
        if (!st) st = check(p + "feed_forward.w1.weight", {E, F});
        if (!st) st = check(p + "feed_forward.w2.weight", {F, E});
        if (!st) st = check(p + "feed_forward.w3.weight", {E, F});
    }
    if (!st) st = check("output_norm.weight", {E});
    if (!st) st = check("output.weight", {E, V});
    return st;
}

}  // namespace velo

// ---------------------------------------------------------------- C ABI

struct velo_gguf {
    velo::GgufFile file;
    mutable std::vector<std::string> names;  // storage for velo_gguf_weights' names (a cache)
};

using velo::fail;

namespace {

void fill_value(const velo::GgufValue& v, velo_gguf_value* out) {
    *out = velo_gguf_value{};
    out->type = (int32_t)v.type;
    out->u = v.u;
    out->i = v.i;
    out->f = v.f;
    if (v.type == 8) {
        out->s = v.s.c_str();
        out->s_len = v.s.size();
    }
    if (v.type == 9) {
        out->u = 0;
        out->array_type = (int32_t)v.u;
        out->array_len = v.arr.size();
    }
}

}  // namespace

extern "C" {

int32_t velo_gguf_open(const char* path, velo_gguf** out) {
    velo::Range nvtx_range("velo.gguf_open");
    velo::clear_last_error();
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    velo_gguf* g = new velo_gguf();
    const int32_t st = velo::gguf_open(path, g->file);
    if (st) {
        delete g;
        return st;
    }
    *out = g;
    return VELO_OK;
}

void velo_gguf_close(velo_gguf* g) { delete g; }

uint32_t velo_gguf_version(const velo_gguf* g) { return g ? g->file.version : 0; }
uint64_t velo_gguf_n_tensors(const velo_gguf* g) { return g ? g->file.tensors.size() : 0; }
uint64_t velo_gguf_n_metadata(const velo_gguf* g) { return g ? g->file.meta.size() : 0; }
uint64_t velo_gguf_data_offset(const velo_gguf* g) { return g ? g->file.data_offset : 0; }

int32_t velo_gguf_metadata(const velo_gguf* g, const char* key, velo_gguf_value* out) {
    velo::clear_last_error();
    if (!g || !key || !out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    auto it = g->file.meta.find(key);
    if (it == g->file.meta.end()) return fail(VELO_ERR_MISSING_META, "missing metadata key: %s", key);
    fill_value(it->second, out);
    return VELO_OK;
}

int32_t velo_gguf_metadata_elem(const velo_gguf* g, const char* key, uint64_t index, velo_gguf_value* out) {
    velo::clear_last_error();
    if (!g || !key || !out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    auto it = g->file.meta.find(key);
    if (it == g->file.meta.end()) return fail(VELO_ERR_MISSING_META, "missing metadata key: %s", key);
    if (it->second.type != 9) return fail(VELO_ERR_INVALID_ARGUMENT, "%s is not an array", key);
    if (index >= it->second.arr.size())
        return fail(VELO_ERR_INVALID_ARGUMENT, "%s[%llu] out of range (%zu elements)", key,
                    (unsigned long long)index, it->second.arr.size());
    fill_value(it->second.arr[(size_t)index], out);
    return VELO_OK;
}

int32_t velo_gguf_tensor_info(const velo_gguf* g, const char* name, velo_gguf_tensor* out) {
    velo::clear_last_error();
    if (!g || !name || !out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    auto it = g->file.tensors.find(name);
    if (it == g->file.tensors.end()) return fail(VELO_ERR_MISSING_TENSOR, "missing tensor: %s", name);
    const velo::GgufTensor& t = it->second;
    *out = velo_gguf_tensor{};
    out->ggml_type = (int32_t)t.ggml_type;
    out->n_dims = (uint32_t)t.shape.size();
    for (size_t d = 0; d < t.shape.size(); ++d) out->shape[d] = t.shape[d];
    out->offset = t.offset;
    out->nbytes = t.nbytes;
    out->data = g->file.data ? g->file.data + t.offset : nullptr;
    return VELO_OK;
}

int32_t velo_gguf_read_model_meta(const velo_gguf* g, velo_gguf_model_meta* out) {
    velo::clear_last_error();
    if (!g || !out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    velo::GgufModelMeta m;
    const int32_t st = velo::gguf_model_meta(g->file, m);
    if (st) return st;
    const uint64_t vals[] = {m.n_vocab, m.n_embd, m.n_layer, m.n_head, m.n_head_kv, m.n_ff, m.head_dim, m.n_ctx};
    for (uint64_t v : vals)
        if (v > 0xffffffffull) return fail(VELO_ERR_INVALID_ARGUMENT, "a model dimension exceeds 32 bits");
    *out = velo_gguf_model_meta{};
    out->struct_size = sizeof(velo_gguf_model_meta);
    out->desc.struct_size = sizeof(velo_model_desc);
    out->desc.n_vocab = (uint32_t)m.n_vocab;
    out->desc.n_embd = (uint32_t)m.n_embd;
    out->desc.n_layer = (uint32_t)m.n_layer;
    out->desc.n_head = (uint32_t)m.n_head;
    out->desc.n_head_kv = (uint32_t)m.n_head_kv;
    out->desc.n_ff = (uint32_t)m.n_ff;
    out->desc.head_dim = (uint32_t)m.head_dim;
    out->desc.rope_freq_base = m.rope_freq_base;
    out->desc.norm_eps = m.norm_eps;
    out->n_ctx = (uint32_t)m.n_ctx;
    out->quantization = m.quantization;
    std::strncpy(out->arch, m.arch.c_str(), sizeof(out->arch) - 1);
    return VELO_OK;
}

int32_t velo_gguf_validate(const velo_gguf* g) {
    velo::clear_last_error();
    if (!g) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    velo::GgufModelMeta m;
    int32_t st = velo::gguf_model_meta(g->file, m);
    if (!st) st = velo::gguf_validate(g->file, m);
    return st;
}

int32_t velo_gguf_weights(const velo_gguf* g, velo_weight_desc* out, int32_t cap, int32_t* n) {
    velo::clear_last_error();
    if (!g || !n) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    velo::GgufModelMeta m;
    int32_t st = velo::gguf_model_meta(g->file, m);
    if (!st) st = velo::gguf_validate(g->file, m);
    if (st) return st;
    std::vector<std::string> names = {"token_embd.weight"};
    static const char* per_layer[] = {"attention_norm.weight", "attention.wq.weight", "attention.wk.weight",
                                      "attention.wv.weight",   "attention.wo.weight", "ffn_norm.weight",
                                      "feed_forward.w1.weight", "feed_forward.w2.weight",
                                      "feed_forward.w3.weight"};
    for (uint64_t l = 0; l < m.n_layer; ++l)
        for (const char* s : per_layer) names.push_back("layers." + std::to_string(l) + "." + s);
    names.push_back("output_norm.weight");
    names.push_back("output.weight");
    *n = (int32_t)names.size();
    if (!out) return VELO_OK;
    if (cap < (int32_t)names.size())
        return fail(VELO_ERR_INVALID_ARGUMENT, "out holds %d descriptors, %zu needed", cap, names.size());
    if (g->names != names) g->names = std::move(names);  // equal lists keep earlier pointers valid
    for (size_t k = 0; k < g->names.size(); ++k) {
        const velo::GgufTensor& t = g->file.tensors.at(g->names[k]);
        int32_t dt;
        if (t.ggml_type == 0) dt = VELO_DT_F32;
        else if (t.ggml_type == 1) dt = VELO_DT_F16;
        else if (t.ggml_type == 2) dt = VELO_DT_Q4_0;
        else
            return fail(VELO_ERR_INVALID_ARGUMENT, "tensor %s: ggml type %u is not supported (F32, F16, Q4_0)",
                        t.name.c_str(), t.ggml_type);
        // rows x cols in the tensor's encoding must be exactly its data bytes
        // (the open-time check bounds every product by 2^64)
        uint64_t rows = 1;
        for (size_t d = 1; d < t.shape.size(); ++d) rows *= t.shape[d];
        const uint64_t cols = t.shape.empty() ? 0 : t.shape[0];
        const unsigned __int128 row_bytes = dt == VELO_DT_F32   ? (unsigned __int128)cols * 4
                                            : dt == VELO_DT_F16 ? (unsigned __int128)cols * 2
                                                                : (unsigned __int128)(cols / 32) * 18;
        if ((dt == VELO_DT_Q4_0 && cols % 32) || row_bytes * rows != (unsigned __int128)t.nbytes)
            return fail(VELO_ERR_INVALID_SHAPE, "tensor %s: %llu x %llu elements do not match its %llu bytes",
                        t.name.c_str(), (unsigned long long)rows, (unsigned long long)cols,
                        (unsigned long long)t.nbytes);
        out[k] = velo_weight_desc{g->names[k].c_str(), dt, 0u, g->file.data + t.offset, rows,
                                  t.shape.empty() ? 0 : t.shape[0]};
    }
    return VELO_OK;
}

int32_t velo_cuda_load_gguf(velo_cuda_ctx* ctx, const char* path) {
    velo::clear_last_error();
    if (!ctx) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    velo_gguf* g = nullptr;
    int32_t st = velo_gguf_open(path, &g);
    if (st) return st;
    velo_gguf_model_meta meta;
    st = velo_gguf_read_model_meta(g, &meta);
    int32_t n = 0;
    if (!st) st = velo_gguf_weights(g, nullptr, 0, &n);
    std::vector<velo_weight_desc> w((size_t)n);
    if (!st) st = velo_gguf_weights(g, w.data(), n, &n);
    if (!st) st = velo_cuda_load_model(ctx, &meta.desc, w.data(), n);
    velo_gguf_close(g);
    return st;
}

}  // extern "C"
