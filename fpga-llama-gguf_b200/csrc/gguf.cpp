// GGUF files and the CPU backend's Q4_0x8 repack, for callers that load weights without llama.cpp.
//
// b200q_gguf_open maps a .gguf file read-only and parses its header, metadata and tensor table (GGUF v2 / v3: the
// published layout, little endian: "GGUF", version, tensor count, metadata count, the key/value pairs, the tensor
// infos (name, dims, ggml type, data offset), then the data section at the next multiple of general.alignment,
// default 32). Every length and offset is checked against the file's size before it is used, so a truncated or
// corrupt file is refused with a message instead of read past its end. Tensor data is handed out as pointers into the
// mapping, in the GGUF block bytes b200q_upload_weight takes.
//
// b200q_q4_0x8_to_q4_0 undoes ggml's CPU_REPACK layout of Q4_0 (block_q4_0x8: per group of 8 rows and 32-column
// block, the 8 fp16 scales, then 16 chunks of 8 quant bytes, chunk j holding bytes 8 (j / 8) .. of row j % 8, each
// byte XOR 0x88), as the reference backend does before its own repack (ggml-xrt.cpp:683-710, xrt_gguf): the result
// is the original Q4_0 rows bit for bit.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/b200q.h"
#include "layout.h"

namespace {

// GGUF metadata value types (the published format's ids)
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kStr = 8, kArr = 9, kU64 = 10,
    kI64 = 11, kF64 = 12
};

size_t scalar_size(uint32_t t) {
    switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
    }
}

// bytes per block and elements per block of the ggml types this library reads (others: row bytes 0)
size_t type_row_bytes(uint32_t type, uint64_t ne0) {
    switch (type) {
    case 0: return ne0 * 4;                          // F32
    case 1: return ne0 * 2;                          // F16
    case 2: return ne0 % 32 ? 0 : ne0 / 32 * 18;     // Q4_0
    case 3: return ne0 % 32 ? 0 : ne0 / 32 * 20;     // Q4_1
    case 8: return ne0 % 32 ? 0 : ne0 / 32 * 34;     // Q8_0
    case 13: return ne0 % 256 ? 0 : ne0 / 256 * 176;  // Q5_K
    case 14: return ne0 % 256 ? 0 : ne0 / 256 * 210;  // Q6_K
    default: return 0;
    }
}

struct Kv {
    std::string key;
    uint32_t type = 0;       // value type; for arrays the element type is `arr_type`
    uint32_t arr_type = 0;
    uint64_t count = 1;      // array elements (1 for a scalar / string)
    const uint8_t *value = nullptr;  // scalar bytes, string bytes, or the array's first element
    uint64_t str_len = 0;    // strings: bytes
};

struct Tensor {
    std::string name;
    uint32_t type = 0, n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0, bytes = 0;
};

class Cursor {
  public:
    Cursor(const uint8_t *p, size_t n) : p_(p), n_(n) {}
    bool take(size_t k, const uint8_t **out) {
        if (k > n_ - pos_) return false;
        *out = p_ + pos_;
        pos_ += k;
        return true;
    }
    template <class T> bool get(T *v) {
        const uint8_t *q;
        if (!take(sizeof(T), &q)) return false;
        std::memcpy(v, q, sizeof(T));
        return true;
    }
    bool str(std::string *s, uint64_t max_len) {
        uint64_t len;
        const uint8_t *q;
        if (!get(&len) || len > max_len || !take(len, &q)) return false;
        s->assign(reinterpret_cast<const char *>(q), len);
        return true;
    }
    size_t pos() const { return pos_; }

  private:
    const uint8_t *p_;
    size_t n_, pos_ = 0;
};

}  // namespace

struct b200q_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_off = 0;
    std::vector<Kv> kv;
    std::vector<Tensor> tensors;
};

namespace {

int gfail(char *msg, unsigned len, const char *fmt, ...) {
    if (msg && len) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(msg, len, fmt, ap);
        va_end(ap);
    }
    return B200Q_ERR_ARG;
}

// Reads one metadata value of type t at the cursor into kv (arrays: element type, count, first element).
bool read_value(Cursor &c, uint32_t t, Kv &kv, int depth) {
    kv.type = t;
    if (t == kStr) {
        uint64_t len;
        const uint8_t *q;
        if (!c.get(&len) || !c.take(len, &q)) return false;
        kv.value = q;
        kv.str_len = len;
        return true;
    }
    if (t == kArr) {
        if (depth > 0) return false;  // nested arrays are not part of the format this reader accepts
        uint32_t et;
        uint64_t n;
        if (!c.get(&et) || !c.get(&n)) return false;
        kv.arr_type = et;
        kv.count = n;
        if (et == kStr) {
            for (uint64_t i = 0; i < n; ++i) {
                uint64_t len;
                const uint8_t *q;
                if (!c.get(&len) || !c.take(len, &q)) return false;
                if (i == 0) kv.value = q - 8;  // the first string's length word
            }
            return true;
        }
        const size_t es = scalar_size(et);
        if (es == 0 || n > (uint64_t(1) << 40) / es) return false;
        const uint8_t *q;
        if (!c.take(size_t(n) * es, &q)) return false;
        kv.value = q;
        return true;
    }
    const size_t es = scalar_size(t);
    if (es == 0) return false;
    return c.take(es, &kv.value);
}

}  // namespace

extern "C" {

int b200q_gguf_open(const char *path, b200q_gguf **out, char *err, unsigned err_len) {
    if (err && err_len) err[0] = '\0';
    if (!path || !out) return gfail(err, err_len, "gguf_open: null argument");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return gfail(err, err_len, "gguf_open: cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        return gfail(err, err_len, "gguf_open: %s is too short for a GGUF header", path);
    }
    void *m = mmap(nullptr, size_t(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        ::close(fd);
        return gfail(err, err_len, "gguf_open: cannot map %s", path);
    }
    b200q_gguf *g = new b200q_gguf();
    g->fd = fd;
    g->map = static_cast<const uint8_t *>(m);
    g->size = size_t(st.st_size);
    auto bad = [&](const char *what) {
        gfail(err, err_len, "gguf_open: %s: %s", path, what);
        b200q_gguf_close(g);
        return B200Q_ERR_ARG;
    };
    Cursor c(g->map, g->size);
    const uint8_t *magic = nullptr;
    if (!c.take(4, &magic) || std::memcmp(magic, "GGUF", 4) != 0) return bad("not a GGUF file (magic)");
    uint64_t n_tensors = 0, n_kv = 0;
    if (!c.get(&g->version) || (g->version != 2 && g->version != 3)) return bad("GGUF version is not 2 or 3");
    // a metadata pair takes at least 13 bytes (key length, type, one value byte), a tensor info at least 32
    if (!c.get(&n_tensors) || !c.get(&n_kv) || n_tensors > g->size / 32 || n_kv > g->size / 13)
        return bad("implausible tensor or metadata count");
    g->kv.resize(size_t(n_kv));
    for (Kv &kv : g->kv) {
        uint32_t t;
        if (!c.str(&kv.key, 1 << 16) || !c.get(&t) || !read_value(c, t, kv, 0)) return bad("truncated metadata");
        if (kv.key == "general.alignment") {
            uint32_t a = 0;
            if (t != kU32) return bad("general.alignment is not a uint32");
            std::memcpy(&a, kv.value, 4);
            if (a == 0 || (a & (a - 1))) return bad("general.alignment is not a power of two");
            g->alignment = a;
        }
    }
    g->tensors.resize(size_t(n_tensors));
    for (Tensor &t : g->tensors) {
        if (!c.str(&t.name, 1 << 16) || !c.get(&t.n_dims) || t.n_dims == 0 || t.n_dims > 4)
            return bad("truncated or invalid tensor info");
        for (uint32_t d = 0; d < t.n_dims; ++d)
            if (!c.get(&t.ne[d]) || t.ne[d] == 0 || t.ne[d] > (uint64_t(1) << 40)) return bad("invalid tensor dims");
        if (!c.get(&t.type) || !c.get(&t.offset)) return bad("truncated tensor info");
    }
    g->data_off = (c.pos() + g->alignment - 1) / g->alignment * g->alignment;
    for (Tensor &t : g->tensors) {
        const size_t rb = type_row_bytes(t.type, t.ne[0]);
        if (rb) {
            const uint64_t rows = t.ne[1] * t.ne[2] * t.ne[3];
            t.bytes = rows * rb;
        }
        if (t.offset % g->alignment) return bad("a tensor's data offset is not aligned");
        if (g->data_off > g->size || t.offset > g->size - g->data_off || t.bytes > g->size - g->data_off - t.offset)
            return bad("a tensor's data runs past the end of the file");
    }
    *out = g;
    return 0;
}

void b200q_gguf_close(b200q_gguf *g) {
    if (!g) return;
    if (g->map) munmap(const_cast<uint8_t *>(g->map), g->size);
    if (g->fd >= 0) ::close(g->fd);
    delete g;
}

uint64_t b200q_gguf_n_tensors(const b200q_gguf *g) { return g ? g->tensors.size() : 0; }
uint64_t b200q_gguf_n_kv(const b200q_gguf *g) { return g ? g->kv.size() : 0; }
uint32_t b200q_gguf_version(const b200q_gguf *g) { return g ? g->version : 0; }

int b200q_gguf_tensor(const b200q_gguf *g, uint64_t index, b200q_gguf_tensor_info *out) {
    if (!g || !out || index >= g->tensors.size()) return B200Q_ERR_ARG;
    const Tensor &t = g->tensors[size_t(index)];
    out->name = t.name.c_str();
    out->type = t.type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; ++d) out->ne[d] = t.ne[d];
    out->offset = g->data_off + t.offset;
    out->bytes = t.bytes;
    out->data = t.bytes ? g->map + g->data_off + t.offset : nullptr;
    return 0;
}

int b200q_gguf_find_tensor(const b200q_gguf *g, const char *name, uint64_t *index) {
    if (!g || !name || !index) return B200Q_ERR_ARG;
    for (size_t i = 0; i < g->tensors.size(); ++i)
        if (g->tensors[i].name == name) {
            *index = i;
            return 0;
        }
    return B200Q_ERR_ARG;
}

int b200q_gguf_kv(const b200q_gguf *g, uint64_t index, b200q_gguf_kv_info *out) {
    if (!g || !out || index >= g->kv.size()) return B200Q_ERR_ARG;
    const Kv &kv = g->kv[size_t(index)];
    out->key = kv.key.c_str();
    out->type = kv.type;
    out->array_type = kv.arr_type;
    out->count = kv.count;
    out->value = kv.value;
    out->str_len = kv.str_len;
    return 0;
}

int b200q_gguf_find_kv(const b200q_gguf *g, const char *key, uint64_t *index) {
    if (!g || !key || !index) return B200Q_ERR_ARG;
    for (size_t i = 0; i < g->kv.size(); ++i)
        if (g->kv[i].key == key) {
            *index = i;
            return 0;
        }
    return B200Q_ERR_ARG;
}

int b200q_gguf_get_int(const b200q_gguf *g, const char *key, int64_t *value) {
    uint64_t i;
    if (!value || b200q_gguf_find_kv(g, key, &i) != 0) return B200Q_ERR_ARG;
    const Kv &kv = g->kv[size_t(i)];
    const uint8_t *p = kv.value;
    switch (kv.type) {
    case kU8: *value = *p; return 0;
    case kI8: *value = int8_t(*p); return 0;
    case kBool: *value = *p != 0; return 0;
    case kU16: { uint16_t v; std::memcpy(&v, p, 2); *value = v; return 0; }
    case kI16: { int16_t v; std::memcpy(&v, p, 2); *value = v; return 0; }
    case kU32: { uint32_t v; std::memcpy(&v, p, 4); *value = v; return 0; }
    case kI32: { int32_t v; std::memcpy(&v, p, 4); *value = v; return 0; }
    case kU64: { uint64_t v; std::memcpy(&v, p, 8); if (v > uint64_t(INT64_MAX)) return B200Q_ERR_ARG; *value = int64_t(v); return 0; }
    case kI64: { int64_t v; std::memcpy(&v, p, 8); *value = v; return 0; }
    default: return B200Q_ERR_ARG;
    }
}

int b200q_gguf_get_float(const b200q_gguf *g, const char *key, double *value) {
    uint64_t i;
    if (!value || b200q_gguf_find_kv(g, key, &i) != 0) return B200Q_ERR_ARG;
    const Kv &kv = g->kv[size_t(i)];
    if (kv.type == kF32) {
        float v;
        std::memcpy(&v, kv.value, 4);
        *value = v;
        return 0;
    }
    if (kv.type == kF64) {
        std::memcpy(value, kv.value, 8);
        return 0;
    }
    int64_t iv;
    if (b200q_gguf_get_int(g, key, &iv) != 0) return B200Q_ERR_ARG;
    *value = double(iv);
    return 0;
}

int b200q_q4_0x8_to_q4_0(const void *src, unsigned rows, unsigned cols, void *dst) {
    if (!src || !dst || rows == 0 || rows % 8 || cols == 0 || cols % 32) return B200Q_ERR_ARG;
    const size_t blocks = cols / 32;
    const uint8_t *in = static_cast<const uint8_t *>(src);
    uint8_t *out = static_cast<uint8_t *>(dst);
    for (size_t grp = 0; grp < rows / 8; ++grp) {
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *x8 = in + (grp * blocks + b) * 144;  // 8 scales (16 bytes) + 128 quant bytes
            for (size_t r = 0; r < 8; ++r) {
                uint8_t *blk = out + ((grp * 8 + r) * blocks + b) * 18;
                blk[0] = x8[2 * r];
                blk[1] = x8[2 * r + 1];
                // quant byte k of row r (k < 16) sits in chunk j = 8 (k / 8) + r at position k % 8
                for (size_t k = 0; k < 16; ++k) blk[2 + k] = uint8_t(x8[16 + 8 * (8 * (k / 8) + r) + k % 8] ^ 0x88u);
            }
        }
    }
    return 0;
}

int b200q_upload_gguf_tensor(b200q_ctx *ctx, const b200q_gguf *g, uint64_t index, unsigned block_cols, unsigned flags,
                             uint64_t *w_off) {
    b200q_gguf_tensor_info t;
    if (!ctx || !w_off || b200q_gguf_tensor(g, index, &t) != 0) return B200Q_ERR_ARG;
    if (t.ne[2] != 1 || t.ne[3] != 1 || t.ne[1] > 0xffffffffu || t.ne[0] > 0xffffffffu || !t.data)
        return B200Q_ERR_ARG;
    return b200q_upload_weight_ex(ctx, t.data, unsigned(t.ne[1]), unsigned(t.ne[0]), t.type, block_cols, flags, w_off);
}

}  // extern "C"
