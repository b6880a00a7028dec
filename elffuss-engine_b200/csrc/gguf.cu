// gguf.cu -- GGUF file reader feeding ef_weight_load (host code).
//
// Restates the reference's parser (js/gguf.js): the ggml type table
// (:48-76: name, block size, type size; retired codes rejected), the header
// (:324-352: magic "GGUF", version 2 or 3, big-endian files recognised and
// rejected, tensor count before key count), the key/value section (:354-361:
// non-empty unique keys, value types 0..12, arrays of any scalar or of
// strings), general.alignment (:363-378: uint32, a power of two, default 32),
// the tensor table (:380-428: unique names, at most 4 dimensions, missing
// dimensions = 1, a known live type, ne0 a multiple of the block, every
// offset exactly the running sum of the previous tensors' padded sizes) and
// the data section (:430-438: aligned after the table when there are
// tensors; every tensor inside the file). The file is memory-mapped; tensor
// bytes are handed to ef_weight_load straight from the mapping.
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/elffuss_cuda.h"

namespace {

struct TypeInfo {
    const char *name;
    int block, size;
};
// ggml type codes 0..41 (block 0 = retired or unknown layout)
const TypeInfo kTypes[] = {
    {"F32", 1, 4},     {"F16", 1, 2},       {"Q4_0", 32, 18},   {"Q4_1", 32, 20},    {"Q4_2", 0, 0},
    {"Q4_3", 0, 0},    {"Q5_0", 32, 22},    {"Q5_1", 32, 24},   {"Q8_0", 32, 34},    {"Q8_1", 32, 40},
    {"Q2_K", 256, 84}, {"Q3_K", 256, 110},  {"Q4_K", 256, 144}, {"Q5_K", 256, 176},  {"Q6_K", 256, 210},
    {"Q8_K", 256, 292}, {"IQ2_XXS", 256, 66}, {"IQ2_XS", 256, 74}, {"IQ3_XXS", 256, 98}, {"IQ1_S", 256, 50},
    {"IQ4_NL", 32, 18}, {"IQ3_S", 256, 110}, {"IQ2_S", 256, 82}, {"IQ4_XS", 256, 136}, {"I8", 1, 1},
    {"I16", 1, 2},     {"I32", 1, 4},       {"I64", 1, 8},      {"F64", 1, 8},       {"IQ1_M", 256, 56},
    {"BF16", 1, 2},    {"Q4_0_4_4", 0, 0},  {"Q4_0_4_8", 0, 0}, {"Q4_0_8_8", 0, 0},  {"TQ1_0", 256, 54},
    {"TQ2_0", 256, 66}, {"IQ4_NL_4_4", 0, 0}, {"IQ4_NL_4_8", 0, 0}, {"IQ4_NL_8_8", 0, 0}, {"MXFP4", 32, 17},
    {"NVFP4", 64, 36}, {"Q1_0", 128, 18},   {"Q2_0", 64, 18},
};
constexpr int kNumTypes = sizeof(kTypes) / sizeof(kTypes[0]);
const int kValueSize[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};   // GGUF value types 0..12
constexpr uint32_t kMaxVersion = 3;
constexpr uint32_t kMaxDims = 4;
constexpr uint64_t kMaxName = 64;
constexpr uint64_t kMaxString = 1ull << 30;

const TypeInfo *type_info(int code) {
    if (code >= 0 && code < kNumTypes) return &kTypes[code];
    static const TypeInfo pq2 = {"PQ2_0", 128, 34}, ptq1 = {"PTQ1_0", 128, 28};   // third-party codes
    if (code == 142) return &pq2;
    if (code == 143) return &ptq1;
    return nullptr;
}

struct Meta {
    std::string key;
    int type;              // value type
    int elem_type = -1;    // arrays: element type
    uint64_t count = 1;    // arrays: element count
    uint64_t at = 0;       // file offset of the value (arrays: of the first element)
    std::string str;       // string values
};

struct Tensor {
    std::string name;
    int type;
    int n_dims;
    int64_t dims[4];
    uint64_t offset, bytes;
};

}  // namespace

struct ef_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0, alignment = 32;
    uint64_t data_start = 0;
    std::vector<Meta> meta;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> by_name, by_key;
};

namespace {

struct Reader {
    const uint8_t *p;
    size_t size, pos = 0;
    char *err;
    size_t errlen;
    bool fail(const char *fmt, ...) {
        if (err && errlen) {
            va_list ap;
            va_start(ap, fmt);
            int n = snprintf(err, errlen, "GGUF: ");
            if (n > 0 && (size_t)n < errlen) vsnprintf(err + n, errlen - n, fmt, ap);
            va_end(ap);
        }
        return false;
    }
    bool need(uint64_t n, const char *what) {
        if (n > size - pos) return fail("file truncated reading %s", what);
        return true;
    }
    bool u32(uint32_t &v, const char *what) {
        if (!need(4, what)) return false;
        memcpy(&v, p + pos, 4);
        pos += 4;
        return true;
    }
    bool i32(int32_t &v, const char *what) {
        if (!need(4, what)) return false;
        memcpy(&v, p + pos, 4);
        pos += 4;
        return true;
    }
    bool u64(uint64_t &v, const char *what) {
        if (!need(8, what)) return false;
        memcpy(&v, p + pos, 8);
        pos += 8;
        return true;
    }
    bool str(std::string &s, const char *what) {
        uint64_t n;
        if (!u64(n, what)) return false;
        if (n > kMaxString) return fail("%s: string of %llu bytes", what, (unsigned long long)n);
        if (!need(n, what)) return fail("%s: string longer than the file", what);
        s.assign(reinterpret_cast<const char *>(p + pos), (size_t)n);
        pos += n;
        return true;
    }
};

uint64_t pad(uint64_t x, uint64_t n) { return x + (n - x % n) % n; }

bool parse(ef_gguf *g, char *err, size_t errlen) {
    Reader r{g->map, g->size, 0, err, errlen};
    if (g->size < 4 || memcmp(g->map, "GGUF", 4) != 0) return r.fail("not a GGUF file (bad magic)");
    r.pos = 4;
    uint32_t version;
    if (!r.u32(version, "version")) return false;
    if (version != 0 && version % 65536 == 0) return r.fail("big-endian file (version %u): not supported", version);
    if (version == 0 || version > kMaxVersion) return r.fail("unsupported version %u", version);
    if (version == 1) return r.fail("GGUFv1 is not supported");
    g->version = version;
    uint64_t n_tensors, n_kv;
    if (!r.u64(n_tensors, "tensor count") || !r.u64(n_kv, "key count")) return false;
    if (n_tensors > g->size || n_kv > g->size) return r.fail("counts larger than the file");
    for (uint64_t i = 0; i < n_kv; i++) {
        Meta m;
        if (!r.str(m.key, "key")) return false;
        if (m.key.empty()) return r.fail("empty key at position %llu", (unsigned long long)i);
        if (g->by_key.count(m.key)) return r.fail("duplicate key '%s'", m.key.c_str());
        int32_t t;
        if (!r.i32(t, "value type")) return false;
        if (t < 0 || t > 12) return r.fail("'%s' has an invalid type %d", m.key.c_str(), t);
        m.type = t;
        if (t == 8) {                                   // string
            m.at = r.pos;
            if (!r.str(m.str, m.key.c_str())) return false;
        } else if (t == 9) {                            // array
            int32_t et;
            if (!r.i32(et, "array type") || !r.u64(m.count, "array length")) return false;
            if (et < 0 || et > 12 || et == 9) return r.fail("'%s': bad array element type %d", m.key.c_str(), et);
            m.elem_type = et;
            m.at = r.pos;
            if (et == 8) {
                if (m.count > (r.size - r.pos) / 8) return r.fail("'%s': string array larger than the file",
                                                                  m.key.c_str());
                std::string s;
                for (uint64_t j = 0; j < m.count; j++)
                    if (!r.str(s, m.key.c_str())) return false;
            } else {
                const uint64_t sz = (uint64_t)kValueSize[et];
                if (m.count > (r.size - r.pos) / sz) return r.fail("'%s': array larger than the file", m.key.c_str());
                r.pos += m.count * sz;
            }
        } else {
            m.at = r.pos;
            if (!r.need(kValueSize[t], m.key.c_str())) return false;
            r.pos += kValueSize[t];
        }
        g->by_key[m.key] = (int64_t)g->meta.size();
        g->meta.push_back(std::move(m));
    }
    auto al = g->by_key.find("general.alignment");
    if (al != g->by_key.end()) {
        const Meta &m = g->meta[al->second];
        if (m.type != 4) return r.fail("general.alignment must be uint32");
        uint32_t a;
        memcpy(&a, g->map + m.at, 4);
        if (a == 0 || (a & (a - 1))) return r.fail("alignment %u is not a power of 2", a);
        g->alignment = a;
    }
    uint64_t expected = 0;
    for (uint64_t i = 0; i < n_tensors; i++) {
        Tensor t;
        if (!r.str(t.name, "tensor name")) return false;
        if (t.name.size() >= kMaxName) return r.fail("tensor name too long (%zu bytes)", t.name.size());
        if (g->by_name.count(t.name)) return r.fail("duplicate tensor name '%s'", t.name.c_str());
        uint32_t nd;
        if (!r.u32(nd, "dimension count")) return false;
        if (nd > kMaxDims) return r.fail("'%s' has %u dimensions (at most %u)", t.name.c_str(), nd, kMaxDims);
        t.n_dims = (int)nd;
        for (int j = 0; j < 4; j++) t.dims[j] = 1;
        for (uint32_t j = 0; j < nd; j++) {
            uint64_t ne;
            if (!r.u64(ne, "dimension")) return false;
            if ((int64_t)ne < 0) return r.fail("'%s' has a negative dimension", t.name.c_str());
            t.dims[j] = (int64_t)ne;
        }
        int32_t ty;
        if (!r.i32(ty, "tensor type") || !r.u64(t.offset, "tensor offset")) return false;
        const TypeInfo *ti = type_info(ty);
        if (!ti) return r.fail("'%s' uses an unknown type %d", t.name.c_str(), ty);
        if (ti->block == 0) return r.fail("'%s' uses the retired type %s", t.name.c_str(), ti->name);
        if (t.dims[0] % ti->block) return r.fail("'%s': ne0=%lld is not a multiple of the %s block",
                                                 t.name.c_str(), (long long)t.dims[0], ti->name);
        t.type = ty;
        unsigned __int128 nb = (unsigned __int128)(t.dims[0] / ti->block) * (unsigned)ti->size;
        for (int j = 1; j < 4; j++) nb *= (unsigned __int128)t.dims[j];
        if (nb > (unsigned __int128)g->size) return r.fail("'%s' is larger than the file", t.name.c_str());
        t.bytes = (uint64_t)nb;
        if (t.offset != expected)
            return r.fail("'%s' is at offset %llu, expected %llu", t.name.c_str(), (unsigned long long)t.offset,
                          (unsigned long long)expected);
        expected = pad(expected + t.bytes, g->alignment);
        g->by_name[t.name] = (int64_t)g->tensors.size();
        g->tensors.push_back(std::move(t));
    }
    g->data_start = n_tensors > 0 ? pad(r.pos, g->alignment) : r.pos;
    uint64_t last = 0;
    for (const Tensor &t : g->tensors) last = t.offset + t.bytes > last ? t.offset + t.bytes : last;
    if (g->data_start + last > g->size)
        return r.fail("tensor data runs past the end of the file (%llu of %zu bytes)",
                      (unsigned long long)(g->data_start + last), g->size);
    return true;
}

}  // namespace

extern "C" {

int ef_gguf_open(const char *path, ef_gguf **out, char *err, size_t errlen) {
    if (err && errlen) err[0] = 0;
    if (!path || !out) return EF_ERR_INVALID;
    *out = nullptr;
    ef_gguf *g = new ef_gguf();
    g->fd = open(path, O_RDONLY);
    if (g->fd < 0) {
        if (err && errlen) snprintf(err, errlen, "GGUF: cannot open %s: %s", path, strerror(errno));
        delete g;
        return EF_ERR_INVALID;
    }
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size <= 0) {
        if (err && errlen) snprintf(err, errlen, "GGUF: empty or unreadable file %s", path);
        close(g->fd);
        delete g;
        return EF_ERR_INVALID;
    }
    g->size = (size_t)st.st_size;
    void *m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        if (err && errlen) snprintf(err, errlen, "GGUF: cannot map %s: %s", path, strerror(errno));
        close(g->fd);
        delete g;
        return EF_ERR_INVALID;
    }
    g->map = (const uint8_t *)m;
    if (!parse(g, err, errlen)) {
        ef_gguf_close(g);
        return EF_ERR_SHAPE;
    }
    *out = g;
    return EF_OK;
}

int ef_gguf_close(ef_gguf *g) {
    if (!g) return EF_ERR_INVALID;
    if (g->map) munmap((void *)g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return EF_OK;
}

int ef_gguf_header(const ef_gguf *g, uint32_t *version, uint32_t *alignment, uint64_t *data_start,
                   int64_t *n_tensors, int64_t *n_meta) {
    if (!g) return EF_ERR_INVALID;
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (data_start) *data_start = g->data_start;
    if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
    if (n_meta) *n_meta = (int64_t)g->meta.size();
    return EF_OK;
}

int ef_gguf_tensor(const ef_gguf *g, int64_t i, const char **name, int *type, int *n_dims, int64_t *dims,
                   uint64_t *file_offset, uint64_t *bytes) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return EF_ERR_RANGE;
    const Tensor &t = g->tensors[(size_t)i];
    if (name) *name = t.name.c_str();
    if (type) *type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int j = 0; j < 4; j++) dims[j] = t.dims[j];
    if (file_offset) *file_offset = g->data_start + t.offset;
    if (bytes) *bytes = t.bytes;
    return EF_OK;
}

int64_t ef_gguf_find_tensor(const ef_gguf *g, const char *name) {
    if (!g || !name) return -1;
    auto it = g->by_name.find(name);
    return it == g->by_name.end() ? -1 : it->second;
}

const void *ef_gguf_tensor_data(const ef_gguf *g, int64_t i) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return nullptr;
    return g->map + g->data_start + g->tensors[(size_t)i].offset;
}

int64_t ef_gguf_find_key(const ef_gguf *g, const char *key) {
    if (!g || !key) return -1;
    auto it = g->by_key.find(key);
    return it == g->by_key.end() ? -1 : it->second;
}

int ef_gguf_meta(const ef_gguf *g, int64_t i, const char **key, int *type, int *elem_type, uint64_t *count,
                 const void **value) {
    if (!g || i < 0 || i >= (int64_t)g->meta.size()) return EF_ERR_RANGE;
    const Meta &m = g->meta[(size_t)i];
    if (key) *key = m.key.c_str();
    if (type) *type = m.type;
    if (elem_type) *elem_type = m.elem_type;
    if (count) *count = m.type == 8 ? (uint64_t)m.str.size() : m.count;
    if (value) *value = m.type == 8 ? (const void *)m.str.data() : (const void *)(g->map + m.at);
    return EF_OK;
}

int ef_gguf_load_weight(ef_ctx *ctx, const ef_gguf *g, const char *name, ef_weight **out) {
    if (!ctx || !g || !name || !out) return EF_ERR_INVALID;
    const int64_t i = ef_gguf_find_tensor(g, name);
    if (i < 0) return EF_ERR_RANGE;
    const Tensor &t = g->tensors[(size_t)i];
    const int64_t k = t.dims[0], rows = t.dims[1] * t.dims[2] * t.dims[3];
    return ef_weight_load(ctx, t.type, g->map + g->data_start + t.offset, rows, k, out);
}

}  // extern "C"
