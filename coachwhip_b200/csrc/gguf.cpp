// GGUF reader: expert banks and a layer's dense tensors straight from a model file.
//
//   reference  candle-core's gguf_file.rs (vendor/candle-core/src/quantized/gguf_file.rs:28-76
//              versioned magic and length prefixes, 130-150 strings, 319-360 values, 469-563
//              Content::read: header, metadata, tensor infos, alignment, data offset) and the
//              resident bank input of ExpertStore::new (crates/engine/src/experts.rs:697-717),
//              which slices blk.L.ffn_{gate,up,down}_exps tensors of shape (E, n, k) per expert.
//
// The file is mapped read-only; a tensor's descriptor points into the mapping, so
// cwx_bank_create copies the bytes from the page cache to the device with no host copy.
// Format (little-endian): magic "GGUF" (either byte order of the u32 is accepted, as candle
// does), u32 version 1..3, tensor count and metadata count (u32 in version 1, else u64),
// metadata entries (string key, u32 value type, value), tensor infos (string name, u32 dims,
// dims x (u32 | u64) ne innermost first, u32 ggml type, u64 offset). Strings are a length and
// bytes, trailing NULs dropped. Tensor data starts at the header's end rounded up to the
// alignment: general.alignment when it is an 8/16/32-bit integer (signed ones when >= 0), else 32.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "cwx_common.cuh"

namespace {

enum : uint32_t {
    GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
    GV_STRING = 8, GV_ARRAY = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};
// dense ggml types read by cwx_gguf_tensor_f32
enum : uint32_t { GT_F32 = 0, GT_F16 = 1, GT_BF16 = 30 };

constexpr uint64_t MAX_COUNT = 1ull << 30;  // strings, arrays, header counts (candle's limits)
constexpr int MAX_DEPTH = 64;
constexpr uint32_t MAX_DIMS = 4;

struct TensorInfo {
    uint32_t type;
    std::vector<uint64_t> ne;  // innermost first
    uint64_t offset;           // from the data section's start
};

struct Meta {
    uint32_t type;
    uint64_t u;      // integer value (signed ones sign-extended)
    double f;        // F32 / F64
    std::string s;   // STRING
};

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool v1 = false;  // version 1: u32 lengths
    bool ok = true;
    const char* why = "truncated";
    uint64_t left() const { return (uint64_t)(end - p); }
    template <typename T>
    T get() {
        T v{};
        if (!ok || left() < sizeof(T)) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    uint64_t len() { return v1 ? (uint64_t)get<uint32_t>() : get<uint64_t>(); }
    void bad(const char* w) {
        if (ok) why = w;
        ok = false;
    }
    std::string str() {
        const uint64_t n = len();
        if (!ok) return {};
        if (n > MAX_COUNT || n > left()) {
            bad("string longer than the file");
            return {};
        }
        size_t m = (size_t)n;
        while (m && p[m - 1] == 0) --m;
        std::string s((const char*)p, m);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if (!ok) return;
        if (n > left()) bad("value longer than the file");
        else p += n;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case GV_U8: case GV_I8: case GV_BOOL: return 1;
        case GV_U16: case GV_I16: return 2;
        case GV_U32: case GV_I32: case GV_F32: return 4;
        case GV_U64: case GV_I64: case GV_F64: return 8;
        default: return 0;
    }
}

// One metadata value of type t: scalars and strings into m, arrays skipped after validation.
void read_value(Cursor& c, uint32_t t, Meta& m, int depth) {
    if (depth > MAX_DEPTH) return c.bad("metadata nested too deep");
    m.type = t;
    switch (t) {
        case GV_U8: m.u = c.get<uint8_t>(); break;
        case GV_I8: m.u = (uint64_t)(int64_t)c.get<int8_t>(); break;
        case GV_U16: m.u = c.get<uint16_t>(); break;
        case GV_I16: m.u = (uint64_t)(int64_t)c.get<int16_t>(); break;
        case GV_U32: m.u = c.get<uint32_t>(); break;
        case GV_I32: m.u = (uint64_t)(int64_t)c.get<int32_t>(); break;
        case GV_U64: m.u = c.get<uint64_t>(); break;
        case GV_I64: m.u = (uint64_t)c.get<int64_t>(); break;
        case GV_F32: m.f = c.get<float>(); break;
        case GV_F64: m.f = c.get<double>(); break;
        case GV_BOOL:
            m.u = c.get<uint8_t>();
            if (m.u > 1) c.bad("bool value other than 0 or 1");
            break;
        case GV_STRING: m.s = c.str(); break;
        case GV_ARRAY: {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.len();
            if (!c.ok) return;
            if (n > MAX_COUNT) return c.bad("array too long");
            const size_t es = scalar_size(et);
            if (es) {
                if (n * es > c.left()) return c.bad("array longer than the file");
                if (et == GV_BOOL)
                    for (uint64_t i = 0; i < n; ++i)
                        if (c.p[i] > 1) return c.bad("bool value other than 0 or 1");
                c.skip(n * es);
            } else if (et == GV_STRING || et == GV_ARRAY) {
                Meta e;
                for (uint64_t i = 0; i < n && c.ok; ++i) read_value(c, et, e, depth + 1);
            } else {
                c.bad("unknown metadata value type");
            }
            break;
        }
        default: c.bad("unknown metadata value type");
    }
}

bool is_int(uint32_t t) {
    return t == GV_U8 || t == GV_I8 || t == GV_U16 || t == GV_I16 || t == GV_U32 || t == GV_I32 || t == GV_U64 ||
           t == GV_I64;
}

float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t b;
    if (e == 31) b = s | 0x7f800000u | (m << 13);
    else if (e) b = s | ((e + 112) << 23) | (m << 13);
    else if (!m) b = s;
    else {  // subnormal: m * 2^-24, exact in f32
        float v = (float)m * (1.0f / 16777216.0f);
        memcpy(&b, &v, 4);
        b |= s;
    }
    float f;
    memcpy(&f, &b, 4);
    return f;
}

}  // namespace

struct cwx_gguf {
    void* map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_offset = 0;  // file offset of the tensor data section
    std::map<std::string, TensorInfo> tensors;
    std::map<std::string, Meta> meta;
};

using namespace cwx;

namespace {

int find_tensor(const cwx_gguf* g, const char* name, const TensorInfo** t, const char* who) {
    if (!g || !name) return fail(CWX_EINVAL, "%s: null argument", who);
    auto it = g->tensors.find(name);
    if (it == g->tensors.end()) return fail(CWX_EINVAL, "%s: no tensor named %s", who, name);
    *t = &it->second;
    return CWX_OK;
}

uint64_t elems(const TensorInfo& t) {
    uint64_t n = 1;
    for (uint64_t d : t.ne) n *= d;
    return n;
}

// Bytes of tensor t, or 0 when its type is not one this library reads.
uint64_t tensor_bytes(const TensorInfo& t) {
    if (t.type == GT_F32) return elems(t) * 4;
    if (t.type == GT_F16 || t.type == GT_BF16) return elems(t) * 2;
    const int be = fmt_block_elems((int)t.type), bb = fmt_block_bytes((int)t.type);
    if (!be || t.ne.empty() || t.ne[0] % (uint64_t)be) return 0;
    return elems(t) / be * bb;
}

int in_file(const cwx_gguf* g, const TensorInfo& t, uint64_t bytes, const char* name, const char* who) {
    const uint64_t at = g->data_offset + t.offset;
    if (t.offset > g->size || at > g->size || bytes > g->size - at)
        return fail(CWX_EINVAL, "%s: %s lies outside the file", who, name);
    return CWX_OK;
}

}  // namespace

extern "C" int cwx_gguf_close(cwx_gguf* g) {
    if (!g) return CWX_OK;
    if (g->map) munmap(g->map, g->size);
    delete g;
    return CWX_OK;
}

extern "C" int cwx_gguf_open(const char* path, cwx_gguf** out) {
    if (!path || !out) return fail(CWX_EINVAL, "cwx_gguf_open: null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(CWX_EINVAL, "cwx_gguf_open: cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 16) {
        close(fd);
        return fail(CWX_EINVAL, "cwx_gguf_open: %s: too short for a GGUF header", path);
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return fail(CWX_EINVAL, "cwx_gguf_open: cannot map %s", path);
    cwx_gguf* g = new cwx_gguf();
    g->map = m;
    g->size = (size_t)st.st_size;
    Cursor c{(const uint8_t*)m, (const uint8_t*)m + g->size};
    auto bad = [&](const char* what) {
        cwx_gguf_close(g);
        return fail(CWX_EINVAL, "cwx_gguf_open: %s: %s", path, what);
    };
    const uint32_t magic = c.get<uint32_t>();
    if (magic != 0x46554747u && magic != 0x47475546u) return bad("bad magic (not a GGUF file)");
    g->version = c.get<uint32_t>();
    if (g->version < 1 || g->version > 3) return bad("unsupported GGUF version");
    c.v1 = g->version == 1;
    const uint64_t n_tensors = c.len(), n_kv = c.len();
    if (!c.ok || n_tensors > MAX_COUNT || n_kv > MAX_COUNT) return bad("header counts out of range");
    const uint64_t pre = c.v1 ? 4 : 8;  // smallest entries: key + type + 1 byte; name + dims + type + offset
    if (n_kv * (pre + 5) + n_tensors * (pre + 16) > c.left()) return bad("header counts larger than the file");
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        if (!c.ok) break;
        Meta v;
        read_value(c, t, v, 0);
        if (c.ok) g->meta[std::move(key)] = std::move(v);
    }
    if (!c.ok) return bad(c.why);
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        std::string name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (!c.ok) break;
        if (nd > MAX_DIMS) return bad("tensor with more than 4 dimensions");
        TensorInfo ti;
        for (uint32_t d = 0; d < nd; ++d) ti.ne.push_back(c.v1 ? (uint64_t)c.get<uint32_t>() : c.get<uint64_t>());
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        if (c.ok) g->tensors[std::move(name)] = std::move(ti);
    }
    if (!c.ok) return bad(c.why);
    auto al = g->meta.find("general.alignment");
    if (al != g->meta.end()) {
        const Meta& a = al->second;
        const bool narrow = a.type == GV_U8 || a.type == GV_U16 || a.type == GV_U32 ||
                            ((a.type == GV_I8 || a.type == GV_I16 || a.type == GV_I32) && (int64_t)a.u >= 0);
        if (narrow) g->alignment = a.u;
        if (!g->alignment) return bad("general.alignment is 0");
    }
    const uint64_t head = (uint64_t)(c.p - (const uint8_t*)m);
    g->data_offset = (head + g->alignment - 1) / g->alignment * g->alignment;
    *out = g;
    return CWX_OK;
}

extern "C" int cwx_gguf_info(const cwx_gguf* g, int32_t* version, int64_t* n_tensors, int64_t* alignment,
                             int64_t* data_offset) {
    if (!g) return fail(CWX_EINVAL, "cwx_gguf_info: null file");
    if (version) *version = (int32_t)g->version;
    if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
    if (alignment) *alignment = (int64_t)g->alignment;
    if (data_offset) *data_offset = (int64_t)g->data_offset;
    return CWX_OK;
}

extern "C" int cwx_gguf_tensor_info(const cwx_gguf* g, const char* name, int32_t* ggml_type, int32_t* n_dims,
                                    int64_t* ne, int64_t* offset) {
    const TensorInfo* t;
    if (int rc = find_tensor(g, name, &t, "cwx_gguf_tensor_info")) return rc;
    if (ggml_type) *ggml_type = (int32_t)t->type;
    if (n_dims) *n_dims = (int32_t)t->ne.size();
    if (ne)
        for (size_t d = 0; d < MAX_DIMS; ++d) ne[d] = d < t->ne.size() ? (int64_t)t->ne[d] : 1;
    if (offset) *offset = (int64_t)(g->data_offset + t->offset);
    return CWX_OK;
}

extern "C" int cwx_gguf_tensor(const cwx_gguf* g, const char* name, cwx_matrix_desc* out) {
    const TensorInfo* t;
    if (int rc = find_tensor(g, name, &t, "cwx_gguf_tensor")) return rc;
    if (!out) return fail(CWX_EINVAL, "cwx_gguf_tensor: null argument");
    if (t->ne.size() < 2 || t->ne.size() > 3)
        return fail(CWX_EUNSUPPORTED, "cwx_gguf_tensor: %s has %zu dimensions, not 2 or 3", name, t->ne.size());
    const int be = fmt_block_elems((int)t->type), bb = fmt_block_bytes((int)t->type);
    if (!be) return fail(CWX_EUNSUPPORTED, "cwx_gguf_tensor: %s has ggml type %u, not an expert format", name, t->type);
    const uint64_t k = t->ne[0], n = t->ne[1], e = t->ne.size() == 3 ? t->ne[2] : 1;
    if (k % (uint64_t)be) return fail(CWX_EINVAL, "cwx_gguf_tensor: %s rows are not whole blocks", name);
    const uint64_t bpe = n * (k / be) * bb;
    if (int rc = in_file(g, *t, bpe * e, name, "cwx_gguf_tensor")) return rc;
    out->ggml_type = (int32_t)t->type;
    out->n = (int64_t)n;
    out->k = (int64_t)k;
    out->n_experts = (int64_t)e;
    out->bytes_per_expert = (int64_t)bpe;
    out->host_ptr = (const uint8_t*)g->map + g->data_offset + t->offset;
    return CWX_OK;
}

extern "C" int cwx_bank_from_gguf(int device, const cwx_gguf* g, const char* name, int64_t first, int64_t n_experts,
                                  cwx_bank** out) {
    cwx_matrix_desc d;
    if (int rc = cwx_gguf_tensor(g, name, &d)) return rc;
    if (n_experts < 0) n_experts = d.n_experts - first;
    if (first < 0 || n_experts <= 0 || first + n_experts > d.n_experts)
        return fail(CWX_EINVAL, "cwx_bank_from_gguf: experts [%lld, %lld) outside %s's %lld", (long long)first,
                    (long long)(first + n_experts), name, (long long)d.n_experts);
    d.host_ptr = (const uint8_t*)d.host_ptr + first * d.bytes_per_expert;
    d.n_experts = n_experts;
    return cwx_bank_create(device, &d, out);
}

extern "C" int cwx_gguf_tensor_f32(const cwx_gguf* g, const char* name, float* out, int64_t n) {
    const TensorInfo* t;
    if (int rc = find_tensor(g, name, &t, "cwx_gguf_tensor_f32")) return rc;
    if (!out) return fail(CWX_EINVAL, "cwx_gguf_tensor_f32: null output");
    if (t->type != GT_F32 && t->type != GT_F16 && t->type != GT_BF16)
        return fail(CWX_EUNSUPPORTED, "cwx_gguf_tensor_f32: %s has ggml type %u, not F32/F16/BF16", name, t->type);
    const uint64_t ne = elems(*t);
    if ((uint64_t)n != ne)
        return fail(CWX_EINVAL, "cwx_gguf_tensor_f32: %s has %llu elements, not %lld", name,
                    (unsigned long long)ne, (long long)n);
    if (int rc = in_file(g, *t, tensor_bytes(*t), name, "cwx_gguf_tensor_f32")) return rc;
    const uint8_t* src = (const uint8_t*)g->map + g->data_offset + t->offset;
    if (t->type == GT_F32) {
        memcpy(out, src, ne * 4);
    } else {
        for (uint64_t i = 0; i < ne; ++i) {
            uint16_t h;
            memcpy(&h, src + 2 * i, 2);
            if (t->type == GT_F16) {
                out[i] = f16_to_f32(h);
            } else {
                const uint32_t b = (uint32_t)h << 16;
                memcpy(out + i, &b, 4);
            }
        }
    }
    return CWX_OK;
}

extern "C" int cwx_gguf_meta_int(const cwx_gguf* g, const char* key, int64_t* out) {
    if (!g || !key || !out) return fail(CWX_EINVAL, "cwx_gguf_meta_int: null argument");
    auto it = g->meta.find(key);
    if (it == g->meta.end() || !is_int(it->second.type))
        return fail(CWX_EINVAL, "cwx_gguf_meta_int: no integer metadata %s", key);
    *out = (int64_t)it->second.u;
    return CWX_OK;
}

extern "C" int cwx_gguf_meta_f64(const cwx_gguf* g, const char* key, double* out) {
    if (!g || !key || !out) return fail(CWX_EINVAL, "cwx_gguf_meta_f64: null argument");
    auto it = g->meta.find(key);
    if (it == g->meta.end() || (it->second.type != GV_F32 && it->second.type != GV_F64))
        return fail(CWX_EINVAL, "cwx_gguf_meta_f64: no float metadata %s", key);
    *out = it->second.f;
    return CWX_OK;
}

extern "C" int cwx_gguf_meta_str(const cwx_gguf* g, const char* key, char* buf, int64_t cap, int64_t* len) {
    if (!g || !key) return fail(CWX_EINVAL, "cwx_gguf_meta_str: null argument");
    auto it = g->meta.find(key);
    if (it == g->meta.end() || it->second.type != GV_STRING)
        return fail(CWX_EINVAL, "cwx_gguf_meta_str: no string metadata %s", key);
    const std::string& s = it->second.s;
    if (len) *len = (int64_t)s.size();
    if (buf && cap > 0) {
        const size_t m = s.size() < (size_t)(cap - 1) ? s.size() : (size_t)(cap - 1);
        memcpy(buf, s.data(), m);
        buf[m] = 0;
    }
    return CWX_OK;
}
