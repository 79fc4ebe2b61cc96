// GGUF container reader (include/stbl_gguf.h).  Host code only.
//
// Layout read (GGUF v2/v3, little endian): magic "GGUF", u32 version, u64 tensor count, u64 metadata
// count; the metadata records (u64-length key string, u32 value type, value); the tensor records
// (name string, u32 dimension count, u64 dims innermost first, u32 type, u64 data offset); the data
// section at the next multiple of `general.alignment` (32 when absent), tensor offsets relative to
// it.  The reference parses the same table (stbl/gguf.cpp:58-99); this reader bounds-checks every
// field against the mapping and refuses what it cannot size instead of reading on.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "stbl_gguf.h"

namespace {

// metadata value types
enum : uint32_t { V_U8, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64, V_COUNT };

uint64_t scalar_bytes(uint32_t t) {
    switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: throw std::runtime_error("metadata value type " + std::to_string(t) + " is not a scalar");
    }
}

// (elements per block, bytes per block) of a tensor type, or {0, 0} when unknown
std::pair<uint64_t, uint64_t> block_of(uint32_t type) {
    switch (type) {
    case STBL_GGUF_F32: return {1, 4};
    case STBL_GGUF_F16: case STBL_GGUF_BF16: return {1, 2};
    case STBL_GGUF_I8: case STBL_GGUF_STBL_E4M3: case STBL_GGUF_STBL_E8M0: return {1, 1};
    case STBL_GGUF_Q8_0: return {32, 34};
    case STBL_GGUF_MXFP4: return {32, 17};
    default: return {0, 0};
    }
}

// bounded reads from the mapping
struct Cursor {
    const uint8_t *base, *p, *end;
    void need(uint64_t n, const char *what) const {
        if ((uint64_t)(end - p) < n) throw std::runtime_error(std::string("file ends inside ") + what);
    }
    template <class T>
    T take(const char *what) {
        need(sizeof(T), what);
        T v;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str(const char *what) {
        const uint64_t n = take<uint64_t>(what);
        need(n, what);
        std::string s(reinterpret_cast<const char *>(p), n);
        p += n;
        return s;
    }
    void skip_value(uint32_t t, int depth) {
        if (depth > 8) throw std::runtime_error("metadata arrays nested too deeply");
        if (t == V_STR) {
            str("a metadata string");
        } else if (t == V_ARR) {
            const uint32_t et = take<uint32_t>("a metadata array");
            const uint64_t n = take<uint64_t>("a metadata array");
            if (et >= V_COUNT) throw std::runtime_error("metadata array of unknown type " + std::to_string(et));
            if (et == V_STR || et == V_ARR) {
                for (uint64_t i = 0; i < n; i++) skip_value(et, depth + 1);
            } else {
                const uint64_t b = scalar_bytes(et);
                if (n > (uint64_t)(end - p) / b) throw std::runtime_error("file ends inside a metadata array");
                p += n * b;
            }
        } else if (t < V_COUNT) {
            const uint64_t b = scalar_bytes(t);
            need(b, "a metadata value");
            p += b;
        } else {
            throw std::runtime_error("metadata value of unknown type " + std::to_string(t));
        }
    }
};

}  // namespace

struct stbl_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    struct Kv {
        std::string key;
        uint32_t type;
        uint64_t at;  // file offset of the value
    };
    std::vector<Kv> kv;
    std::unordered_map<std::string, size_t> kv_index;
    struct Tensor {
        std::string name;
        uint32_t type, n_dims;
        uint64_t dims[4];
        uint64_t offset, nbytes;
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> tensor_index;

    ~stbl_gguf() {
        if (map) munmap(const_cast<uint8_t *>(map), size);
        if (fd >= 0) ::close(fd);
    }

    void parse() {
        Cursor c{map, map, map + size};
        if (c.take<uint32_t>("the header") != 0x46554747u) throw std::runtime_error("not a GGUF file (magic)");
        version = c.take<uint32_t>("the header");
        if (version != 2 && version != 3)
            throw std::runtime_error("GGUF version " + std::to_string(version) + " is not supported (2 or 3)");
        const uint64_t n_tensors = c.take<uint64_t>("the header"), n_kv = c.take<uint64_t>("the header");
        // each record takes at least 12 (metadata) / 24 (tensor) bytes: bounds the reservations
        if (n_kv > size / 12 || n_tensors > size / 24) throw std::runtime_error("record counts exceed the file");
        kv.reserve(n_kv);
        for (uint64_t i = 0; i < n_kv; i++) {
            Kv r;
            r.key = c.str("a metadata key");
            r.type = c.take<uint32_t>("a metadata record");
            r.at = (uint64_t)(c.p - map);
            if (r.key == "general.alignment") {
                if (r.type != V_U32) throw std::runtime_error("general.alignment is not a u32");
                uint32_t a;
                c.need(4, "general.alignment");
                memcpy(&a, c.p, 4);
                if (a == 0) throw std::runtime_error("general.alignment is 0");
                alignment = a;
            }
            c.skip_value(r.type, 0);
            if (kv_index.count(r.key)) throw std::runtime_error("metadata key " + r.key + " appears twice");
            kv_index[r.key] = kv.size();
            kv.push_back(std::move(r));
        }
        tensors.reserve(n_tensors);
        for (uint64_t i = 0; i < n_tensors; i++) {
            Tensor t{};
            t.name = c.str("a tensor name");
            t.n_dims = c.take<uint32_t>("a tensor record");
            if (t.n_dims == 0 || t.n_dims > 4)
                throw std::runtime_error("tensor " + t.name + " has " + std::to_string(t.n_dims) + " dimensions (1-4)");
            uint64_t n = 1;
            for (int d = 0; d < 4; d++) t.dims[d] = 1;
            for (uint32_t d = 0; d < t.n_dims; d++) {
                t.dims[d] = c.take<uint64_t>("a tensor record");
                if (t.dims[d] != 0 && n > UINT64_MAX / t.dims[d]) throw std::runtime_error("tensor " + t.name + " is too large");
                n *= t.dims[d];
            }
            t.type = c.take<uint32_t>("a tensor record");
            t.offset = c.take<uint64_t>("a tensor record");
            const auto blk = block_of(t.type);
            if (!blk.first) throw std::runtime_error("tensor " + t.name + ": unsupported type " + std::to_string(t.type));
            if (n % blk.first) throw std::runtime_error("tensor " + t.name + ": element count not a multiple of its block");
            if (n / blk.first > UINT64_MAX / blk.second) throw std::runtime_error("tensor " + t.name + " is too large");
            t.nbytes = n / blk.first * blk.second;
            if (tensor_index.count(t.name)) throw std::runtime_error("tensor " + t.name + " appears twice");
            tensor_index[t.name] = tensors.size();
            tensors.push_back(std::move(t));
        }
        const uint64_t header = (uint64_t)(c.p - map);
        const uint64_t data = (header + alignment - 1) / alignment * alignment;
        for (auto &t : tensors) {
            if (t.offset > size || data > size - t.offset || t.nbytes > size - t.offset - data)
                throw std::runtime_error("tensor " + t.name + " ends past the end of the file");
            t.offset += data;
        }
    }

    const Kv *find_kv(const char *key, uint32_t type) const {
        auto it = kv_index.find(key ? key : "");
        if (it == kv_index.end()) return nullptr;
        const Kv &r = kv[it->second];
        return r.type == type ? &r : nullptr;
    }

    void fill(const Tensor &t, stbl_gguf_tensor *o) const {
        o->name = t.name.c_str();
        o->type = t.type;
        o->n_dims = t.n_dims;
        for (int d = 0; d < 4; d++) o->dims[d] = t.dims[d];
        o->offset = t.offset;
        o->nbytes = t.nbytes;
        o->data = map + t.offset;
    }
};

extern "C" {

int stbl_gguf_open(const char *path, stbl_gguf **out, char *err, int errlen) {
    stbl_gguf *g = new stbl_gguf();
    try {
        if (!path || !out) throw std::runtime_error("null argument");
        g->fd = ::open(path, O_RDONLY);
        if (g->fd < 0) throw std::runtime_error(std::string("cannot open ") + path + ": " + strerror(errno));
        struct stat st;
        if (fstat(g->fd, &st) != 0) throw std::runtime_error(std::string("cannot stat ") + path);
        g->size = (uint64_t)st.st_size;
        if (g->size < 24) throw std::runtime_error("file too short for a GGUF header");
        void *m = mmap(nullptr, g->size, PROT_READ, MAP_SHARED, g->fd, 0);
        if (m == MAP_FAILED) throw std::runtime_error(std::string("cannot map ") + path);
        g->map = static_cast<const uint8_t *>(m);
        g->parse();
        *out = g;
        return 0;
    } catch (const std::exception &e) {
        if (err && errlen > 0) {
            strncpy(err, e.what(), (size_t)errlen - 1);
            err[errlen - 1] = 0;
        }
        delete g;
        if (out) *out = nullptr;
        return -1;
    }
}

void stbl_gguf_close(stbl_gguf *g) { delete g; }

int stbl_gguf_info(const stbl_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *n_kv, uint64_t *n_tensors) {
    if (!g) return -1;
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (n_kv) *n_kv = g->kv.size();
    if (n_tensors) *n_tensors = g->tensors.size();
    return 0;
}

int stbl_gguf_tensor_at(const stbl_gguf *g, uint64_t i, stbl_gguf_tensor *t) {
    if (!g || !t || i >= g->tensors.size()) return -1;
    g->fill(g->tensors[i], t);
    return 0;
}

int stbl_gguf_find(const stbl_gguf *g, const char *name, stbl_gguf_tensor *t) {
    if (!g || !name || !t) return -1;
    auto it = g->tensor_index.find(name);
    if (it == g->tensor_index.end()) return -1;
    g->fill(g->tensors[it->second], t);
    return 0;
}

int stbl_gguf_kv_at(const stbl_gguf *g, uint64_t i, const char **key, uint32_t *type) {
    if (!g || i >= g->kv.size()) return -1;
    if (key) *key = g->kv[i].key.c_str();
    if (type) *type = g->kv[i].type;
    return 0;
}

int stbl_gguf_u32(const stbl_gguf *g, const char *key, uint32_t *v) {
    const stbl_gguf::Kv *r = g ? g->find_kv(key, V_U32) : nullptr;
    if (!r || !v) return -1;
    memcpy(v, g->map + r->at, 4);
    return 0;
}

int stbl_gguf_f32(const stbl_gguf *g, const char *key, float *v) {
    const stbl_gguf::Kv *r = g ? g->find_kv(key, V_F32) : nullptr;
    if (!r || !v) return -1;
    memcpy(v, g->map + r->at, 4);
    return 0;
}

int64_t stbl_gguf_uints(const stbl_gguf *g, const char *key, uint64_t *v, int64_t cap) {
    const stbl_gguf::Kv *r = g ? g->find_kv(key, V_ARR) : nullptr;
    if (!r) return -1;
    uint32_t et;
    uint64_t n;
    memcpy(&et, g->map + r->at, 4);
    memcpy(&n, g->map + r->at + 4, 8);
    if (et != V_U32 && et != V_U64) return -1;
    const uint8_t *p = g->map + r->at + 12;
    for (uint64_t i = 0; i < n && (int64_t)i < cap; i++) {
        if (et == V_U32) {
            uint32_t x;
            memcpy(&x, p + 4 * i, 4);
            v[i] = x;
        } else {
            memcpy(&v[i], p + 8 * i, 8);
        }
    }
    return (int64_t)n;
}

int64_t stbl_gguf_str(const stbl_gguf *g, const char *key, char *buf, int64_t cap) {
    const stbl_gguf::Kv *r = g ? g->find_kv(key, V_STR) : nullptr;
    if (!r) return -1;
    uint64_t n;
    memcpy(&n, g->map + r->at, 8);
    if (buf && cap > 0) {
        const uint64_t k = n < (uint64_t)(cap - 1) ? n : (uint64_t)(cap - 1);
        memcpy(buf, g->map + r->at + 8, k);
        buf[k] = 0;
    }
    return (int64_t)n;
}

}  // extern "C"
