// gguf.cu -- reading the MoE tensors of a GPT-OSS GGUF file straight into a
// context (host code).
//
// The file is mapped read-only; the header, metadata and tensor index are
// parsed with bounds-checked reads (GGUF v2/v3, little-endian, as
// internal/gguf/reader.go:300-410 reads them), and every tensor's data range is
// checked against the file size.  amoe_upload_layer_gguf then hands pointers
// into the mapping to amoe_upload_layer, which copies the MXFP4 expert bytes to
// the device and repacks them there: nothing is decoded on the host.  Small
// f16/bf16 vectors (norm, router, biases) are widened to f32 first.
#include "../../include/amoe.h"
#include "amoe_internal.cuh"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <limits>
#include <map>
#include <string>
#include <vector>

struct amoe_gguf {
    int fd = -1;
    const uint8_t *base = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    struct Value {
        uint32_t type = 0;  // GGUF metadata value type
        uint64_t u = 0;     // integers (two's complement for signed types)
        double f = 0.0;     // floats
        std::string s;      // strings
        uint64_t count = 0; // arrays: element count
    };
    struct Tensor {
        uint32_t type = 0;
        std::vector<uint64_t> shape;  // shape[0] varies fastest
        int64_t offset = 0;           // absolute, in the file
        int64_t bytes = 0;
    };
    std::map<std::string, Value> meta;
    std::map<std::string, Tensor> tensors;
};

namespace {

using amoe::set_thread_error;

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};

// Bounds-checked little-endian reader over the mapping.
struct Cursor {
    const uint8_t *p, *end;
    std::string err;
    bool need(size_t n) {
        if ((size_t)(end - p) < n) {
            if (err.empty()) err = "truncated header";
            return false;
        }
        return true;
    }
    template <typename T>
    bool get(T *v) {
        if (!need(sizeof(T))) return false;
        std::memcpy(v, p, sizeof(T));
        p += sizeof(T);
        return true;
    }
    bool str(std::string *s) {
        uint64_t n = 0;
        if (!get(&n) || !need(n)) return false;
        s->assign(reinterpret_cast<const char *>(p), (size_t)n);
        p += n;
        return true;
    }
};

bool scalar_size(uint32_t type, size_t *n) {
    switch (type) {
        case kU8: case kI8: case kBool: *n = 1; return true;
        case kU16: case kI16: *n = 2; return true;
        case kU32: case kI32: case kF32: *n = 4; return true;
        case kU64: case kI64: case kF64: *n = 8; return true;
        default: return false;
    }
}

bool read_scalar(Cursor &c, uint32_t type, amoe_gguf::Value *v) {
    size_t n = 0;
    if (!scalar_size(type, &n)) {
        c.err = "unknown metadata value type " + std::to_string(type);
        return false;
    }
    if (!c.need(n)) return false;
    uint64_t raw = 0;
    std::memcpy(&raw, c.p, n);
    c.p += n;
    v->type = type;
    switch (type) {
        case kI8: v->u = (uint64_t)(int64_t)(int8_t)raw; break;
        case kI16: v->u = (uint64_t)(int64_t)(int16_t)raw; break;
        case kI32: v->u = (uint64_t)(int64_t)(int32_t)raw; break;
        case kF32: {
            float f;
            std::memcpy(&f, &raw, 4);
            v->f = f;
            break;
        }
        case kF64: {
            double d;
            std::memcpy(&d, &raw, 8);
            v->f = d;
            break;
        }
        case kBool:
            if (raw > 1) {
                c.err = "invalid boolean value " + std::to_string(raw);
                return false;
            }
            v->u = raw;
            break;
        default: v->u = raw;
    }
    return true;
}

bool read_value(Cursor &c, amoe_gguf::Value *v) {
    uint32_t type = 0;
    if (!c.get(&type)) return false;
    if (type == kString) {
        v->type = type;
        return c.str(&v->s);
    }
    if (type != kArray) return read_scalar(c, type, v);
    uint32_t et = 0;
    uint64_t n = 0;
    if (!c.get(&et) || !c.get(&n)) return false;
    if (et == kArray) {
        c.err = "nested arrays are not valid GGUF metadata";
        return false;
    }
    v->type = kArray;
    v->count = n;
    for (uint64_t i = 0; i < n; ++i) {  // walk the elements (only the count is kept)
        if (et == kString) {
            uint64_t len = 0;
            if (!c.get(&len) || !c.need(len)) return false;
            c.p += len;
        } else {
            size_t sz = 0;
            if (!scalar_size(et, &sz)) {
                c.err = "unknown metadata value type " + std::to_string(et);
                return false;
            }
            if (n > (uint64_t)(c.end - c.p) / sz) {
                c.err = "truncated header";
                return false;
            }
            c.p += sz * n;
            break;
        }
    }
    return true;
}

// Encoded bytes of a tensor (reader.go:419-500): block formats need whole blocks.
bool encoded_size(uint32_t type, const std::vector<uint64_t> &shape, int64_t *bytes, std::string *err) {
    unsigned __int128 n = 1;
    for (uint64_t d : shape) {
        n *= d;
        if (n > (unsigned __int128)std::numeric_limits<int64_t>::max()) {
            *err = "tensor is too large";
            return false;
        }
    }
    const uint64_t e = (uint64_t)n;
    const uint64_t kMax = (uint64_t)std::numeric_limits<int64_t>::max();
    // every size must fit int64 (reader.go:429-466): "encoded tensor size overflows int64"
    auto scalar = [&](uint64_t width) {
        if (e > kMax / width) {
            *err = "encoded tensor size overflows int64";
            return false;
        }
        *bytes = (int64_t)(e * width);
        return true;
    };
    auto blocks = [&](uint64_t per, uint64_t bytes_per, const char *what) {
        if (e % per) {
            *err = std::string(what) + " element count must be divisible by " + std::to_string(per);
            return false;
        }
        if (e / per > kMax / bytes_per) {
            *err = "encoded tensor size overflows int64";
            return false;
        }
        *bytes = (int64_t)(e / per * bytes_per);
        return true;
    };
    switch (type) {
        case AMOE_GGUF_F32: return scalar(4);
        case AMOE_GGUF_F16: case AMOE_GGUF_BF16: return scalar(2);
        case AMOE_GGUF_MXFP4: return blocks(32, 17, "MXFP4");
        case AMOE_GGUF_Q8_0: return blocks(32, 34, "Q8_0");
        case AMOE_GGUF_Q4_0: return blocks(32, 18, "Q4_0");
        case AMOE_GGUF_Q4_K: return blocks(256, 144, "Q4_K");
        case AMOE_GGUF_Q5_K: return blocks(256, 176, "Q5_K");
        case AMOE_GGUF_Q6_K: return blocks(256, 210, "Q6_K");
        default: *err = "unsupported tensor type " + std::to_string(type); return false;
    }
}

bool parse(amoe_gguf *g, std::string *err) {
    Cursor c{g->base, g->base + g->size, ""};
    char magic[4];
    if (!c.need(4)) {
        *err = "read magic: file too short";
        return false;
    }
    std::memcpy(magic, c.p, 4);
    c.p += 4;
    if (std::memcmp(magic, "GGUF", 4) != 0) {
        *err = "invalid magic";
        return false;
    }
    uint64_t ntensor = 0, nmeta = 0;
    if (!c.get(&g->version) || !(g->version == 2 || g->version == 3)) {
        *err = c.err.empty() ? "unsupported version " + std::to_string(g->version) + ": want 2 or 3" : c.err;
        return false;
    }
    if (!c.get(&ntensor) || !c.get(&nmeta)) {
        *err = c.err;
        return false;
    }
    for (uint64_t i = 0; i < nmeta; ++i) {
        std::string key;
        amoe_gguf::Value v;
        if (!c.str(&key)) {
            *err = "read metadata key " + std::to_string(i) + ": " + c.err;
            return false;
        }
        if (g->meta.count(key)) {
            *err = "duplicate metadata key \"" + key + "\"";
            return false;
        }
        if (!read_value(c, &v)) {
            *err = "read metadata \"" + key + "\": " + c.err;
            return false;
        }
        g->meta.emplace(key, std::move(v));
    }
    std::vector<std::pair<std::string, uint64_t>> rel;
    for (uint64_t i = 0; i < ntensor; ++i) {
        std::string name;
        uint32_t nd = 0, type = 0;
        uint64_t off = 0;
        if (!c.str(&name) || !c.get(&nd)) {
            *err = "read tensor " + std::to_string(i) + ": " + c.err;
            return false;
        }
        if (g->tensors.count(name)) {
            *err = "duplicate tensor \"" + name + "\"";
            return false;
        }
        if (nd > 64) {
            *err = "tensor \"" + name + "\" has unreasonable dimension count " + std::to_string(nd);
            return false;
        }
        amoe_gguf::Tensor t;
        t.shape.resize(nd);
        for (uint32_t j = 0; j < nd; ++j)
            if (!c.get(&t.shape[j])) {
                *err = "tensor \"" + name + "\" shape: " + c.err;
                return false;
            }
        if (!c.get(&type) || !c.get(&off)) {
            *err = "tensor \"" + name + "\": " + c.err;
            return false;
        }
        t.type = type;
        std::string why;
        if (!encoded_size(type, t.shape, &t.bytes, &why)) {
            *err = "tensor \"" + name + "\": " + why;
            return false;
        }
        rel.emplace_back(name, off);
        g->tensors.emplace(name, std::move(t));
    }
    uint64_t alignment = 32;
    auto it = g->meta.find("general.alignment");
    if (it != g->meta.end()) {
        const auto &v = it->second;
        const bool uint_like = v.type == kU8 || v.type == kU16 || v.type == kU32 || v.type == kU64 ||
                               ((v.type == kI8 || v.type == kI16 || v.type == kI32 || v.type == kI64) && (int64_t)v.u >= 0);
        if (!uint_like || v.u == 0 || v.u > (uint64_t)std::numeric_limits<int64_t>::max()) {
            *err = "invalid general.alignment";
            return false;
        }
        alignment = v.u;
    }
    const uint64_t header_end = (uint64_t)(c.p - g->base);
    if (header_end > std::numeric_limits<uint64_t>::max() - (alignment - 1)) {
        *err = "tensor data offset exceeds file size";
        return false;
    }
    const uint64_t data = (header_end + alignment - 1) / alignment * alignment;
    if (data > g->size) {
        *err = "tensor data offset exceeds file size";
        return false;
    }
    for (auto &r : rel) {
        auto &t = g->tensors[r.first];
        if (r.second > g->size - data || (uint64_t)t.bytes > g->size - data - r.second) {
            *err = "tensor \"" + r.first + "\" data range exceeds file size";
            return false;
        }
        t.offset = (int64_t)(data + r.second);
    }
    return true;
}

bool is_int(uint32_t t) { return t == kU8 || t == kI8 || t == kU16 || t == kI16 || t == kU32 || t == kI32 || t == kU64 || t == kI64; }
bool is_signed(uint32_t t) { return t == kI8 || t == kI16 || t == kI32 || t == kI64; }

// Integer metadata (numberInt in reader.go): any integer type; unsigned values
// above INT64_MAX are rejected.  0 = found, 1 = absent, -1 = wrong type.
int meta_int(const amoe_gguf *g, const std::string &key, int64_t *out) {
    auto it = g->meta.find(key);
    if (it == g->meta.end()) return 1;
    const auto &v = it->second;
    if (!is_int(v.type)) return -1;
    if (!is_signed(v.type) && v.u > (uint64_t)std::numeric_limits<int64_t>::max()) return -1;
    *out = (int64_t)v.u;
    return 0;
}

int meta_float(const amoe_gguf *g, const std::string &key, double *out) {
    auto it = g->meta.find(key);
    if (it == g->meta.end()) return 1;
    if (it->second.type != kF32 && it->second.type != kF64) return -1;
    *out = it->second.f;
    return 0;
}

const amoe_gguf::Tensor *find(const amoe_gguf *g, const std::string &name) {
    auto it = g->tensors.find(name);
    return it == g->tensors.end() ? nullptr : &it->second;
}

std::string shape_str(const std::vector<uint64_t> &s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? " " : "") + std::to_string(s[i]);
    return r + "]";
}

// A tensor with exactly this GGUF shape (checkShape, internal/model/gptoss/tensor.go:116-127).
const amoe_gguf::Tensor *shaped(const amoe_gguf *g, const std::string &name, std::vector<uint64_t> want,
                                std::string *err) {
    const amoe_gguf::Tensor *t = find(g, name);
    if (!t) {
        *err = "gptoss: tensor \"" + name + "\" not found";
        return nullptr;
    }
    if (t->shape != want) {
        *err = "gptoss: tensor \"" + name + "\" shape " + shape_str(t->shape) + ", want GGUF shape " + shape_str(want);
        return nullptr;
    }
    return t;
}

float half_bits_to_float(uint16_t h, bool bf16) {
    if (bf16) {
        const uint32_t u = (uint32_t)h << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t u;
    if (e == 31) u = s | 0x7f800000u | (m << 13);  // inf / NaN
    else if (e) u = s | ((e + 112) << 23) | (m << 13);
    else if (!m) u = s;
    else {  // subnormal half: normalize
        int ee = -1;
        uint32_t mm = m;
        do {
            ++ee;
            mm <<= 1;
        } while (!(mm & 1024));
        u = s | ((uint32_t)(112 - ee) << 23) | ((mm & 1023) << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// An f32 view of a small vector tensor: the mapped bytes for F32, else widened into `buf`.
const float *f32_view(const amoe_gguf *g, const amoe_gguf::Tensor *t, std::vector<float> &buf, std::string *err,
                      const std::string &name) {
    const uint8_t *p = g->base + t->offset;
    size_t n = 1;
    for (uint64_t d : t->shape) n *= (size_t)d;
    switch (t->type) {
        case AMOE_GGUF_F32:
            if (reinterpret_cast<uintptr_t>(p) % 4 == 0) return reinterpret_cast<const float *>(p);
            buf.resize(n);
            std::memcpy(buf.data(), p, n * 4);
            return buf.data();
        case AMOE_GGUF_F16:
        case AMOE_GGUF_BF16: {
            buf.resize(n);
            for (size_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                buf[i] = half_bits_to_float(h, t->type == AMOE_GGUF_BF16);
            }
            return buf.data();
        }
        default:
            *err = "gptoss: tensor \"" + name + "\" type " + std::to_string(t->type) +
                   ": the MoE block takes f32, f16 or bf16 vectors";
            return nullptr;
    }
}

}  // namespace

namespace amoe {

// The head (loadResidentWeights, internal/model/gptoss/weights.go:19-33): output_norm.weight [H],
// and output.weight [H, V], or token_embd.weight [H, V] when the file has no output.weight (the
// reference then reuses the embeddings as the lm head).  The lm head stays in its GGUF encoding
// (F32, F16 or BF16; the reference decodes those three, tensor.go:137-144).
int gguf_head(const amoe_gguf *g, int H, int V, GgufHead *out, std::string *err) {
    const uint64_t h = H, v = V;
    const amoe_gguf::Tensor *n = shaped(g, "output_norm.weight", {h}, err);
    if (!n || !(out->norm = f32_view(g, n, out->buf, err, "output_norm.weight"))) return -1;
    const char *name = find(g, "output.weight") ? "output.weight" : "token_embd.weight";
    const amoe_gguf::Tensor *w = shaped(g, name, {h, v}, err);
    if (!w) return -1;
    if (w->type != AMOE_GGUF_F32 && w->type != AMOE_GGUF_F16 && w->type != AMOE_GGUF_BF16) {
        *err = std::string("gptoss: tensor \"") + name + "\" type " + std::to_string(w->type) +
               ": the lm head takes f32, f16 or bf16";
        return -1;
    }
    out->type = (int)w->type;
    const uint8_t *p = g->base + w->offset;
    const size_t align = w->type == AMOE_GGUF_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(p) % align == 0) {
        out->lm_head = p;
    } else {
        out->head_buf.assign(p, p + w->bytes);
        out->lm_head = out->head_buf.data();
    }
    return 0;
}

// Layer `layer`'s MoE tensors (loadDecoderLayer, internal/model/gptoss/weights.go:35-124, its MoE
// part): the post-attention norm (ffn_norm or post_attention_norm), the router, and the experts
// either fused (ffn_gate_up_exps, rows interleaving gate and up) or split (ffn_gate_exps +
// ffn_up_exps, interleaved here into the fused row order), plus ffn_down_exps.  Shapes are
// checked exactly as the reference does; the expert tensors must be MXFP4.
int gguf_layer(const amoe_gguf *g, int layer, int H, int I, int E, GgufLayer *L, std::string *err) {
    const std::string pre = "blk." + std::to_string(layer) + ".";
    const uint64_t h = H, i = I, e = E;
    auto vec = [&](const std::string &name, std::vector<uint64_t> shape, std::vector<float> &buf) -> const float * {
        const amoe_gguf::Tensor *t = shaped(g, pre + name, shape, err);
        return t ? f32_view(g, t, buf, err, pre + name) : nullptr;
    };
    auto mxfp4 = [&](const std::string &name, std::vector<uint64_t> shape) -> const uint8_t * {
        const amoe_gguf::Tensor *t = shaped(g, pre + name, shape, err);
        if (!t) return nullptr;
        if (t->type != AMOE_GGUF_MXFP4) {
            *err = "gptoss: tensor \"" + pre + name + "\" type " + std::to_string(t->type) +
                   ": the expert weights must be MXFP4";
            return nullptr;
        }
        return g->base + t->offset;
    };
    const char *norm = find(g, pre + "ffn_norm.weight") ? "ffn_norm.weight" : "post_attention_norm.weight";
    if (!(L->norm = vec(norm, {h}, L->buf[0])) || !(L->router_w = vec("ffn_gate_inp.weight", {h, e}, L->buf[1])) ||
        !(L->router_b = vec("ffn_gate_inp.bias", {e}, L->buf[2])))
        return -1;
    if (find(g, pre + "ffn_gate_up_exps.weight")) {
        if (!(L->gu = mxfp4("ffn_gate_up_exps.weight", {h, 2 * i, e})) ||
            !(L->gu_b = vec("ffn_gate_up_exps.bias", {2 * i, e}, L->buf[3])))
            return -1;
    } else {
        const uint8_t *gate = mxfp4("ffn_gate_exps.weight", {h, i, e});
        const uint8_t *up = gate ? mxfp4("ffn_up_exps.weight", {h, i, e}) : nullptr;
        std::vector<float> gb, ub;
        const float *gbias = up ? vec("ffn_gate_exps.bias", {i, e}, gb) : nullptr;
        const float *ubias = gbias ? vec("ffn_up_exps.bias", {i, e}, ub) : nullptr;
        if (!ubias) return -1;
        const size_t row = (size_t)(H / 32) * 17;
        L->gu_buf.resize((size_t)E * 2 * I * row);
        L->buf[3].resize((size_t)E * 2 * I);
        for (size_t x = 0; x < e; ++x)
            for (size_t r = 0; r < i; ++r) {
                const size_t src = x * i + r, dst = x * 2 * i + 2 * r;
                std::memcpy(&L->gu_buf[dst * row], gate + src * row, row);
                std::memcpy(&L->gu_buf[(dst + 1) * row], up + src * row, row);
                L->buf[3][dst] = gbias[src];
                L->buf[3][dst + 1] = ubias[src];
            }
        L->gu = L->gu_buf.data();
        L->gu_b = L->buf[3].data();
    }
    if (!(L->dn = mxfp4("ffn_down_exps.weight", {i, h, e})) || !(L->dn_b = vec("ffn_down_exps.bias", {h, e}, L->buf[4])))
        return -1;
    return 0;
}

}  // namespace amoe

extern "C" {

int amoe_gguf_open(const char *path, amoe_gguf **out) {
    if (!path || !out) {
        set_thread_error("path and out must not be NULL");
        return AMOE_ERR_INVALID;
    }
    *out = nullptr;
    amoe_gguf *g = new (std::nothrow) amoe_gguf();
    if (!g) {
        set_thread_error("out of host memory");
        return AMOE_ERR_NOMEM;
    }
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        set_thread_error(std::string("gguf: open ") + path + ": " + std::strerror(errno));
        amoe_gguf_close(g);
        return AMOE_ERR_INVALID;
    }
    g->size = (size_t)st.st_size;
    if (g->size > 0) {
        void *m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
        if (m == MAP_FAILED) {
            set_thread_error(std::string("gguf: map ") + path + ": " + std::strerror(errno));
            amoe_gguf_close(g);
            return AMOE_ERR_INVALID;
        }
        g->base = static_cast<const uint8_t *>(m);
    }
    std::string err;
    if (!parse(g, &err)) {
        set_thread_error("gguf: " + err);
        amoe_gguf_close(g);
        return AMOE_ERR_INVALID;
    }
    *out = g;
    return AMOE_OK;
}

void amoe_gguf_close(amoe_gguf *g) {
    if (!g) return;
    if (g->base) munmap(const_cast<uint8_t *>(g->base), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

int amoe_gguf_tensor(const amoe_gguf *g, const char *name, int32_t *type, int32_t *ndims, int64_t *dims,
                     int64_t *offset, int64_t *bytes) {
    if (!g || !name) {
        set_thread_error("gguf and name must not be NULL");
        return AMOE_ERR_INVALID;
    }
    const amoe_gguf::Tensor *t = find(g, name);
    if (!t) {
        set_thread_error(std::string("gguf: tensor \"") + name + "\" not found");
        return AMOE_ERR_INVALID;
    }
    if (type) *type = (int32_t)t->type;
    if (ndims) *ndims = (int32_t)t->shape.size();
    if (dims)
        for (size_t i = 0; i < t->shape.size() && i < 4; ++i) dims[i] = (int64_t)t->shape[i];
    if (offset) *offset = t->offset;
    if (bytes) *bytes = t->bytes;
    return AMOE_OK;
}

int amoe_gguf_moe_config(const amoe_gguf *g, amoe_config *cfg) {
    if (!g || !cfg) {
        set_thread_error("gguf and cfg must not be NULL");
        return AMOE_ERR_INVALID;
    }
    auto arch = g->meta.find("general.architecture");
    if (arch == g->meta.end() || arch->second.type != kString) {
        set_thread_error("gguf: metadata \"general.architecture\" must be a string");
        return AMOE_ERR_INVALID;
    }
    std::string prefix;
    if (arch->second.s == "gptoss") prefix = "gptoss.";
    else if (arch->second.s == "gpt-oss") prefix = "gpt-oss.";
    else {
        set_thread_error("gguf: unsupported architecture \"" + arch->second.s +
                         "\": only gptoss and gpt-oss are supported");
        return AMOE_ERR_INVALID;
    }
    struct Field {
        const char *suffix;
        int32_t *dst;
    } fields[] = {{"embedding_length", &cfg->hidden},
                  {"expert_feed_forward_length", &cfg->intermediate},
                  {"expert_count", &cfg->experts},
                  {"expert_used_count", &cfg->top_k},
                  {"block_count", &cfg->layers}};
    int32_t vals[5];
    for (int i = 0; i < 5; ++i) {
        int64_t v = 0;
        const std::string key = prefix + fields[i].suffix;
        const int rc = meta_int(g, key, &v);
        if (rc == 1) {
            set_thread_error("gguf: missing metadata \"" + key + "\"");
            return AMOE_ERR_INVALID;
        }
        if (rc < 0 || v <= 0 || v > std::numeric_limits<int32_t>::max()) {
            set_thread_error("gguf: metadata \"" + key + "\" must be a positive integer");
            return AMOE_ERR_INVALID;
        }
        vals[i] = (int32_t)v;
    }
    double eps = 0.0;
    const std::string ekey = prefix + "attention.layer_norm_rms_epsilon";
    const int rc = meta_float(g, ekey, &eps);
    if (rc != 0 || !(eps > 0.0) || !std::isfinite(eps)) {
        set_thread_error(rc == 1 ? "gguf: missing metadata \"" + ekey + "\"" : "gguf: invalid RMS norm epsilon");
        return AMOE_ERR_INVALID;
    }
    for (int i = 0; i < 5; ++i) *fields[i].dst = vals[i];
    cfg->rms_eps = (float)eps;
    return AMOE_OK;
}

}  // extern "C"
