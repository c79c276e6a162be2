// GGUF reader: maps a GGUF file (the llama.cpp / ggml model container, the
// format feml's roadmap names as the producer of quantized weights,
// docs/DESIGN.md:282-286 of the reference) read-only and parses its header, key/value
// metadata and tensor table, so that weights can be uploaded straight from
// the mapping into a plan's Weights buffer (feml_b200_buffer_from_host_ptr,
// feml_b200_write) without an intermediate host copy.
//
// Format (public GGUF specification, versions 2 and 3, little-endian):
//   u32 magic "GGUF", u32 version, u64 tensor_count, u64 kv_count,
//   kv_count x { string key, u32 value_type, value },
//   tensor_count x { string name, u32 n_dims, u64 ne[n_dims], u32 ggml_type,
//                    u64 offset (relative to the data section) },
//   padding to `general.alignment` (default 32), then the data section.
//   string = u64 length + bytes (no terminator); array = u32 element type +
//   u64 count + elements.
// Every read is bounds-checked against the file size; a malformed file gives
// FB_ERR_INVALID with the offset of the problem, never an out-of-range read.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "host_common.h"

namespace {

using fb::set_error;

enum : uint32_t {
    GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STRING, GT_ARRAY, GT_U64, GT_I64, GT_F64,
    GT_COUNT
};

size_t scalar_size(uint32_t t) {
    switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
    }
}

// ggml type id -> (block elements, block bytes, feml dtype or -1). Sizes of the
// public ggml type table; ids without an entry are listed with unknown size.
struct GgmlType {
    uint32_t id;
    int64_t blck, bytes;
    int32_t dtype;
};
constexpr GgmlType kGgmlTypes[] = {
    {0, 1, 4, FB_F32},      {1, 1, 2, FB_F16},       {2, 32, 18, FB_Q4_0},   {3, 32, 20, FB_Q4_1},
    {6, 32, 22, FB_Q5_0},   {7, 32, 24, FB_Q5_1},    {8, 32, 34, FB_Q8_0},   {9, 32, 36, FB_Q8_1},
    {10, 256, 84, FB_Q2_K}, {11, 256, 110, FB_Q3_K}, {12, 256, 144, FB_Q4_K}, {13, 256, 176, FB_Q5_K},
    {14, 256, 210, FB_Q6_K}, {15, 256, 292, FB_Q8_K}, {24, 1, 1, FB_I8},    {25, 1, 2, FB_I16},
    {26, 1, 4, FB_I32},     {27, 1, 8, FB_I64},      {28, 1, 8, FB_F64},     {30, 1, 2, -1 /* BF16 */},
};

const GgmlType *ggml_type(uint32_t id) {
    for (const GgmlType &t : kGgmlTypes)
        if (t.id == id) return &t;
    return nullptr;
}

struct Kv {
    std::string key;
    uint32_t type = 0;
    uint32_t elem_type = 0;  // arrays
    uint64_t count = 0;      // arrays: element count; strings: byte length
    uint64_t data = 0;       // file offset of the scalar, the string bytes or the first array element
    std::vector<std::pair<uint64_t, uint64_t>> strs;  // string arrays: (offset, length) per element
};

struct Tensor {
    std::string name;
    uint32_t ggml_type = 0;
    int32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t rel_offset = 0;
    uint64_t nbytes = 0;
    int32_t dtype = -1;
};

class Cursor {
  public:
    Cursor(const uint8_t *base, uint64_t size) : base_(base), size_(size) {}
    uint64_t pos() const { return pos_; }
    bool need(uint64_t n, const char *what) {
        if (n > size_ - pos_) {
            set_error(FB_ERR_INVALID, "gguf: truncated file: %s at offset %llu needs %llu bytes, %llu left", what,
                      (unsigned long long)pos_, (unsigned long long)n, (unsigned long long)(size_ - pos_));
            return false;
        }
        return true;
    }
    template <typename T>
    bool get(T &v, const char *what) {
        if (!need(sizeof(T), what)) return false;
        std::memcpy(&v, base_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return true;
    }
    bool skip(uint64_t n, const char *what) {
        if (!need(n, what)) return false;
        pos_ += n;
        return true;
    }
    // string: (offset, length) of its bytes
    bool str(uint64_t &off, uint64_t &len, const char *what) {
        if (!get(len, what) || !need(len, what)) return false;
        off = pos_;
        pos_ += len;
        return true;
    }

  private:
    const uint8_t *base_;
    uint64_t size_;
    uint64_t pos_ = 0;
};

}  // namespace

struct fb_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_offset = 0;
    std::vector<Kv> kvs;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> kv_index, tensor_index;
};

namespace {

void destroy(fb_gguf *g) {
    if (!g) return;
    if (g->map) munmap(const_cast<uint8_t *>(g->map), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

bool read_value(Cursor &c, uint32_t type, Kv &kv, int depth) {
    if (type == GT_STRING) {
        return c.str(kv.data, kv.count, "string value");
    }
    if (type == GT_ARRAY) {
        if (depth > 0) {
            set_error(FB_ERR_INVALID, "gguf: nested array in key '%s' (offset %llu)", kv.key.c_str(),
                      (unsigned long long)c.pos());
            return false;
        }
        uint64_t n = 0;
        if (!c.get(kv.elem_type, "array type") || !c.get(n, "array length")) return false;
        kv.count = n;
        kv.data = c.pos();
        if (kv.elem_type == GT_STRING) {
            kv.strs.reserve((size_t)std::min<uint64_t>(n, 1u << 20));
            for (uint64_t i = 0; i < n; i++) {
                uint64_t off, len;
                if (!c.str(off, len, "string array element")) return false;
                kv.strs.emplace_back(off, len);
            }
            return true;
        }
        const size_t es = scalar_size(kv.elem_type);
        if (es == 0) {
            set_error(FB_ERR_INVALID, "gguf: key '%s' has arrays of unknown type %u", kv.key.c_str(), kv.elem_type);
            return false;
        }
        if (n > UINT64_MAX / es) {
            set_error(FB_ERR_INVALID, "gguf: key '%s' array length %llu overflows", kv.key.c_str(),
                      (unsigned long long)n);
            return false;
        }
        return c.skip(n * es, "array elements");
    }
    const size_t sz = scalar_size(type);
    if (sz == 0) {
        set_error(FB_ERR_INVALID, "gguf: key '%s' has unknown value type %u", kv.key.c_str(), type);
        return false;
    }
    kv.data = c.pos();
    return c.skip(sz, "scalar value");
}

int parse(fb_gguf *g) {
    Cursor c(g->map, g->size);
    uint32_t magic = 0;
    if (!c.get(magic, "magic")) return FB_ERR_INVALID;
    if (std::memcmp(g->map, "GGUF", 4) != 0)
        return set_error(FB_ERR_INVALID, "gguf: bad magic (not a little-endian GGUF file)");
    if (!c.get(g->version, "version")) return FB_ERR_INVALID;
    if (g->version != 2 && g->version != 3)
        return set_error(FB_ERR_UNSUPPORTED, "gguf: version %u not supported (2 and 3 are)", g->version);
    uint64_t n_tensors = 0, n_kv = 0;
    if (!c.get(n_tensors, "tensor count") || !c.get(n_kv, "kv count")) return FB_ERR_INVALID;
    // every entry takes at least 8 bytes, which bounds the counts by the file size
    if (n_tensors > g->size / 8 || n_kv > g->size / 8)
        return set_error(FB_ERR_INVALID, "gguf: counts (%llu tensors, %llu keys) exceed the file size",
                         (unsigned long long)n_tensors, (unsigned long long)n_kv);
    g->kvs.resize((size_t)n_kv);
    for (uint64_t i = 0; i < n_kv; i++) {
        Kv &kv = g->kvs[(size_t)i];
        uint64_t off, len;
        if (!c.str(off, len, "key")) return FB_ERR_INVALID;
        kv.key.assign(reinterpret_cast<const char *>(g->map + off), (size_t)len);
        if (kv.key.find('\0') != std::string::npos)  // keys are handed out as C strings
            return set_error(FB_ERR_INVALID, "gguf: key %llu contains a NUL byte", (unsigned long long)i);
        if (!c.get(kv.type, "value type") || !read_value(c, kv.type, kv, 0)) return FB_ERR_INVALID;
        if (!g->kv_index.emplace(kv.key, (int64_t)i).second)
            return set_error(FB_ERR_INVALID, "gguf: duplicate key '%s'", kv.key.c_str());
    }
    auto al = g->kv_index.find("general.alignment");
    if (al != g->kv_index.end()) {
        const Kv &kv = g->kvs[(size_t)al->second];
        if (kv.type != GT_U32) return set_error(FB_ERR_INVALID, "gguf: general.alignment is not a u32");
        uint32_t a;
        std::memcpy(&a, g->map + kv.data, 4);
        if (a == 0 || (a & (a - 1)))
            return set_error(FB_ERR_INVALID, "gguf: general.alignment %u is not a power of two", a);
        g->alignment = a;
    }
    g->tensors.resize((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        Tensor &t = g->tensors[(size_t)i];
        uint64_t off, len;
        if (!c.str(off, len, "tensor name")) return FB_ERR_INVALID;
        t.name.assign(reinterpret_cast<const char *>(g->map + off), (size_t)len);
        if (t.name.find('\0') != std::string::npos)  // names are looked up as C strings
            return set_error(FB_ERR_INVALID, "gguf: tensor %llu's name contains a NUL byte", (unsigned long long)i);
        uint32_t nd = 0;
        if (!c.get(nd, "tensor n_dims")) return FB_ERR_INVALID;
        if (nd < 1 || nd > 4)
            return set_error(FB_ERR_UNSUPPORTED, "gguf: tensor '%s' has %u dimensions (1..4 supported)",
                             t.name.c_str(), nd);
        t.n_dims = (int32_t)nd;
        uint64_t elems = 1;
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t ne;
            if (!c.get(ne, "tensor dims")) return FB_ERR_INVALID;
            if (ne == 0 || ne > (uint64_t)INT64_MAX || elems > (uint64_t)INT64_MAX / ne)
                return set_error(FB_ERR_INVALID, "gguf: tensor '%s' dimension %u is %llu", t.name.c_str(), d,
                                 (unsigned long long)ne);
            t.ne[d] = (int64_t)ne;
            elems *= ne;
        }
        if (!c.get(t.ggml_type, "tensor type") || !c.get(t.rel_offset, "tensor offset")) return FB_ERR_INVALID;
        if (t.rel_offset % g->alignment)
            return set_error(FB_ERR_INVALID, "gguf: tensor '%s' offset %llu is not a multiple of the alignment %llu",
                             t.name.c_str(), (unsigned long long)t.rel_offset, (unsigned long long)g->alignment);
        if (const GgmlType *gt = ggml_type(t.ggml_type)) {
            if (t.ne[0] % gt->blck)
                return set_error(FB_ERR_SHAPE, "gguf: tensor '%s' ne[0] %lld is not a multiple of the block %lld",
                                 t.name.c_str(), (long long)t.ne[0], (long long)gt->blck);
            t.nbytes = elems / (uint64_t)gt->blck * (uint64_t)gt->bytes;
            t.dtype = gt->dtype;
        }
        if (!g->tensor_index.emplace(t.name, (int64_t)i).second)
            return set_error(FB_ERR_INVALID, "gguf: duplicate tensor '%s'", t.name.c_str());
    }
    const uint64_t end = c.pos();
    g->data_offset = (end + g->alignment - 1) / g->alignment * g->alignment;
    for (const Tensor &t : g->tensors) {
        const uint64_t start = g->data_offset + t.rel_offset;
        if (start < g->data_offset || start > g->size || t.nbytes > g->size - start)
            return set_error(FB_ERR_INVALID, "gguf: tensor '%s' data [%llu, +%llu) lies outside the file (%llu bytes)",
                             t.name.c_str(), (unsigned long long)start, (unsigned long long)t.nbytes,
                             (unsigned long long)g->size);
    }
    return FB_OK;
}

const Kv *kv_at(const fb_gguf *g, int64_t i) {
    if (!g || i < 0 || i >= (int64_t)g->kvs.size()) {
        set_error(FB_ERR_INVALID, "gguf: no key at index %lld", (long long)i);
        return nullptr;
    }
    return &g->kvs[(size_t)i];
}

}  // namespace

extern "C" {

int feml_b200_gguf_open(const char *path, fb_gguf **out) {
    if (!path || !out) return set_error(FB_ERR_INVALID, "gguf_open: null argument");
    *out = nullptr;
    fb_gguf *g = new fb_gguf();
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) {
        destroy(g);
        return set_error(FB_ERR_INVALID, "gguf_open: cannot open '%s': %s", path, strerror(errno));
    }
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
        destroy(g);
        return set_error(FB_ERR_INVALID, "gguf_open: '%s' is not a GGUF file (too small)", path);
    }
    g->size = (uint64_t)st.st_size;
    void *m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        destroy(g);
        return set_error(FB_ERR_INVALID, "gguf_open: mmap of '%s' failed: %s", path, strerror(errno));
    }
    g->map = static_cast<const uint8_t *>(m);
    const int rc = parse(g);
    if (rc) {
        destroy(g);
        return rc;
    }
    *out = g;
    return FB_OK;
}

int feml_b200_gguf_close(fb_gguf *g) {
    destroy(g);
    return FB_OK;
}

int feml_b200_gguf_info(const fb_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *data_offset,
                        int64_t *n_kv, int64_t *n_tensors) {
    if (!g) return set_error(FB_ERR_INVALID, "gguf_info: null file");
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data_offset;
    if (n_kv) *n_kv = (int64_t)g->kvs.size();
    if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
    return FB_OK;
}

int feml_b200_gguf_tensor(const fb_gguf *g, int64_t index, fb_gguf_tensor *out) {
    if (!g || !out) return set_error(FB_ERR_INVALID, "gguf_tensor: null argument");
    if (index < 0 || index >= (int64_t)g->tensors.size())
        return set_error(FB_ERR_INVALID, "gguf_tensor: no tensor at index %lld", (long long)index);
    const Tensor &t = g->tensors[(size_t)index];
    if (t.name.size() >= sizeof(out->name))
        return set_error(FB_ERR_UNSUPPORTED, "gguf_tensor: name of tensor %lld longer than %zu bytes",
                         (long long)index, sizeof(out->name) - 1);
    std::memset(out, 0, sizeof(*out));
    std::memcpy(out->name, t.name.data(), t.name.size());
    out->dtype = t.dtype;
    out->ggml_type = t.ggml_type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; d++) out->ne[d] = t.ne[d];
    out->offset = g->data_offset + t.rel_offset;
    out->nbytes = t.nbytes;
    return FB_OK;
}

int feml_b200_gguf_find_tensor(const fb_gguf *g, const char *name, int64_t *index) {
    if (!g || !name || !index) return set_error(FB_ERR_INVALID, "gguf_find_tensor: null argument");
    auto it = g->tensor_index.find(name);
    if (it == g->tensor_index.end()) return set_error(FB_ERR_INVALID, "gguf: no tensor named '%s'", name);
    *index = it->second;
    return FB_OK;
}

int feml_b200_gguf_tensor_data(const fb_gguf *g, int64_t index, const void **data) {
    if (!g || !data) return set_error(FB_ERR_INVALID, "gguf_tensor_data: null argument");
    if (index < 0 || index >= (int64_t)g->tensors.size())
        return set_error(FB_ERR_INVALID, "gguf_tensor_data: no tensor at index %lld", (long long)index);
    *data = g->map + g->data_offset + g->tensors[(size_t)index].rel_offset;
    return FB_OK;
}

int feml_b200_gguf_kv(const fb_gguf *g, int64_t index, const char **key, uint32_t *type, uint32_t *elem_type,
                      uint64_t *count) {
    const Kv *kv = kv_at(g, index);
    if (!kv) return FB_ERR_INVALID;
    if (key) *key = kv->key.c_str();
    if (type) *type = kv->type;
    if (elem_type) *elem_type = kv->type == GT_ARRAY ? kv->elem_type : 0;
    if (count) *count = kv->type == GT_ARRAY ? kv->count : (kv->type == GT_STRING ? kv->count : 1);
    return FB_OK;
}

int feml_b200_gguf_find_kv(const fb_gguf *g, const char *key, int64_t *index) {
    if (!g || !key || !index) return set_error(FB_ERR_INVALID, "gguf_find_kv: null argument");
    auto it = g->kv_index.find(key);
    if (it == g->kv_index.end()) return set_error(FB_ERR_INVALID, "gguf: no key '%s'", key);
    *index = it->second;
    return FB_OK;
}

int feml_b200_gguf_kv_int(const fb_gguf *g, int64_t index, int64_t *out) {
    const Kv *kv = kv_at(g, index);
    if (!kv || !out) return kv ? set_error(FB_ERR_INVALID, "gguf_kv_int: null out") : FB_ERR_INVALID;
    const uint8_t *p = g->map + kv->data;
    switch (kv->type) {
    case GT_U8: *out = *p; break;
    case GT_I8: *out = (int8_t)*p; break;
    case GT_BOOL: *out = *p != 0; break;
    case GT_U16: { uint16_t v; std::memcpy(&v, p, 2); *out = v; break; }
    case GT_I16: { int16_t v; std::memcpy(&v, p, 2); *out = v; break; }
    case GT_U32: { uint32_t v; std::memcpy(&v, p, 4); *out = v; break; }
    case GT_I32: { int32_t v; std::memcpy(&v, p, 4); *out = v; break; }
    case GT_I64: { int64_t v; std::memcpy(&v, p, 8); *out = v; break; }
    case GT_U64: {
        uint64_t v;
        std::memcpy(&v, p, 8);
        if (v > (uint64_t)INT64_MAX)
            return set_error(FB_ERR_UNSUPPORTED, "gguf: key '%s' value %llu does not fit int64", kv->key.c_str(),
                             (unsigned long long)v);
        *out = (int64_t)v;
        break;
    }
    default: return set_error(FB_ERR_INVALID, "gguf: key '%s' is not an integer (type %u)", kv->key.c_str(), kv->type);
    }
    return FB_OK;
}

int feml_b200_gguf_kv_float(const fb_gguf *g, int64_t index, double *out) {
    const Kv *kv = kv_at(g, index);
    if (!kv || !out) return kv ? set_error(FB_ERR_INVALID, "gguf_kv_float: null out") : FB_ERR_INVALID;
    const uint8_t *p = g->map + kv->data;
    if (kv->type == GT_F32) {
        float v;
        std::memcpy(&v, p, 4);
        *out = v;
    } else if (kv->type == GT_F64) {
        std::memcpy(out, p, 8);
    } else {
        return set_error(FB_ERR_INVALID, "gguf: key '%s' is not a float (type %u)", kv->key.c_str(), kv->type);
    }
    return FB_OK;
}

int feml_b200_gguf_kv_str(const fb_gguf *g, int64_t index, int64_t elem, const char **s, uint64_t *len) {
    const Kv *kv = kv_at(g, index);
    if (!kv || !s || !len) return kv ? set_error(FB_ERR_INVALID, "gguf_kv_str: null out") : FB_ERR_INVALID;
    if (kv->type == GT_STRING) {
        *s = reinterpret_cast<const char *>(g->map + kv->data);
        *len = kv->count;
        return FB_OK;
    }
    if (kv->type == GT_ARRAY && kv->elem_type == GT_STRING) {
        if (elem < 0 || elem >= (int64_t)kv->strs.size())
            return set_error(FB_ERR_INVALID, "gguf: key '%s' has no element %lld", kv->key.c_str(), (long long)elem);
        *s = reinterpret_cast<const char *>(g->map + kv->strs[(size_t)elem].first);
        *len = kv->strs[(size_t)elem].second;
        return FB_OK;
    }
    return set_error(FB_ERR_INVALID, "gguf: key '%s' is not a string", kv->key.c_str());
}

int feml_b200_gguf_kv_array_data(const fb_gguf *g, int64_t index, const void **data) {
    const Kv *kv = kv_at(g, index);
    if (!kv || !data) return kv ? set_error(FB_ERR_INVALID, "gguf_kv_array_data: null out") : FB_ERR_INVALID;
    if (kv->type != GT_ARRAY || kv->elem_type == GT_STRING)
        return set_error(FB_ERR_INVALID, "gguf: key '%s' is not a numeric array", kv->key.c_str());
    *data = g->map + kv->data;
    return FB_OK;
}

}  // extern "C"
