// gguf_reader.cu — GGUF tensor reader and device upload (host code).
//
// The reference engine loads its weights from GGUF files
// (desktop/engine/src/gguf_loader.cpp, tensors bound in llama_weights.cpp:
// 866-950); the on-disk tensor bytes are the same block_q4_K / block_q6_K
// rows the kernels here stream, so a model's matrices can be uploaded
// unchanged. This parser follows the GGUF v2/v3 layout (vendor/ggml/include/
// gguf.h): magic "GGUF", version, tensor count, KV count; the KV pairs
// (string key, value type, value or typed array); the tensor infos (name,
// n_dims, ne[], ggml type, offset into the data section); the data section
// at the first multiple of general.alignment (default 32) after the infos.
// The file is memory-mapped read-only; every length and offset is checked
// against the file size before use, so a truncated or corrupt file is
// rejected with BH_EINVAL rather than read out of bounds.
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "bh_ctx.cuh"
#include "../../include/bh_q4k.h"

namespace {

enum : uint32_t {
    GT_UINT8 = 0, GT_INT8 = 1, GT_UINT16 = 2, GT_INT16 = 3, GT_UINT32 = 4, GT_INT32 = 5, GT_FLOAT32 = 6,
    GT_BOOL = 7, GT_STRING = 8, GT_ARRAY = 9, GT_UINT64 = 10, GT_INT64 = 11, GT_FLOAT64 = 12, GT_COUNT = 13
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case GT_UINT8: case GT_INT8: case GT_BOOL: return 1;
        case GT_UINT16: case GT_INT16: return 2;
        case GT_UINT32: case GT_INT32: case GT_FLOAT32: return 4;
        case GT_UINT64: case GT_INT64: case GT_FLOAT64: return 8;
        default: return 0;
    }
}

// Bytes of one block and values per block of the ggml types a model file
// holds (vendor/ggml/src/ggml-common.h block layouts).
bool type_block(int t, size_t* bytes, int64_t* values) {
    switch (t) {
        case 0: *bytes = 4; *values = 1; return true;      // F32
        case 1: *bytes = 2; *values = 1; return true;      // F16
        case 30: *bytes = 2; *values = 1; return true;     // BF16
        case 2: *bytes = 18; *values = 32; return true;    // Q4_0
        case 3: *bytes = 20; *values = 32; return true;    // Q4_1
        case 6: *bytes = 22; *values = 32; return true;    // Q5_0
        case 7: *bytes = 24; *values = 32; return true;    // Q5_1
        case 8: *bytes = 34; *values = 32; return true;    // Q8_0
        case 10: *bytes = 84; *values = 256; return true;  // Q2_K
        case 11: *bytes = 110; *values = 256; return true; // Q3_K
        case 12: *bytes = 144; *values = 256; return true; // Q4_K
        case 13: *bytes = 176; *values = 256; return true; // Q5_K
        case 14: *bytes = 210; *values = 256; return true; // Q6_K
        case 15: *bytes = 292; *values = 256; return true; // Q8_K
        default: return false;
    }
}

struct KV {
    std::string key;
    uint32_t type;        // scalar type, GT_STRING, or GT_ARRAY
    uint32_t arr_type;    // element type of an array
    uint64_t arr_n;
    const uint8_t* val;   // the value's bytes in the mapping
};

struct TensorInfo {
    std::string name;
    int type;
    int n_dims;
    int64_t ne[4];
    uint64_t offset;      // from the start of the data section
    uint64_t bytes;       // 0 when the type's block size is unknown
};

}  // namespace

struct bh_gguf {
    int fd = -1;
    const uint8_t* map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    size_t alignment = 32;
    size_t data_off = 0;
    std::vector<KV> kv;
    std::vector<TensorInfo> tensors;
};

namespace {

struct Cursor {
    const uint8_t* p;
    size_t left;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if (left < sizeof(T)) { ok = false; left = 0; return v; }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        left -= sizeof(T);
        return v;
    }
    const uint8_t* take(uint64_t n) {
        if (n > left) { ok = false; left = 0; return nullptr; }
        const uint8_t* r = p;
        p += n;
        left -= n;
        return r;
    }
    bool str(std::string* s) {
        const uint64_t n = get<uint64_t>();
        const uint8_t* b = take(n);
        if (!ok) return false;
        if (s) s->assign(reinterpret_cast<const char*>(b), (size_t)n);
        return true;
    }
};

// Skip (validate) one value of type t; arrays of strings are walked.
bool skip_value(Cursor& c, uint32_t t, KV* kv) {
    if (t == GT_STRING) return c.str(nullptr);
    if (t == GT_ARRAY) {
        const uint32_t at = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (!c.ok || at >= GT_COUNT || at == GT_ARRAY) return false;
        if (kv) { kv->arr_type = at; kv->arr_n = n; }
        if (at == GT_STRING) {
            for (uint64_t i = 0; i < n; ++i)
                if (!c.str(nullptr)) return false;
            return true;
        }
        const size_t es = scalar_size(at);
        if (es == 0 || n > c.left / es) return false;
        c.take(n * es);
        return c.ok;
    }
    const size_t es = scalar_size(t);
    if (es == 0) return false;
    c.take(es);
    return c.ok;
}

int parse(bh_gguf* g) {
    Cursor c{g->map, g->size};
    const uint8_t* magic = c.take(4);
    if (!c.ok || std::memcmp(magic, "GGUF", 4) != 0) return BH_EINVAL;
    g->version = c.get<uint32_t>();
    if (g->version < 2 || g->version > 3) return BH_EINVAL;
    const int64_t n_tensors = c.get<int64_t>();
    const int64_t n_kv = c.get<int64_t>();
    if (!c.ok || n_tensors < 0 || n_kv < 0 || (uint64_t)n_tensors > g->size || (uint64_t)n_kv > g->size)
        return BH_EINVAL;
    g->kv.reserve((size_t)n_kv);
    for (int64_t i = 0; i < n_kv; ++i) {
        KV kv{};
        if (!c.str(&kv.key)) return BH_EINVAL;
        kv.type = c.get<uint32_t>();
        if (!c.ok || kv.type >= GT_COUNT) return BH_EINVAL;
        kv.val = c.p;
        if (!skip_value(c, kv.type, &kv)) return BH_EINVAL;
        if (kv.key == "general.alignment") {
            if (kv.type != GT_UINT32) return BH_EINVAL;
            uint32_t a;
            std::memcpy(&a, kv.val, 4);
            if (a == 0 || (a & (a - 1)) != 0) return BH_EINVAL;
            g->alignment = a;
        }
        g->kv.push_back(std::move(kv));
    }
    g->tensors.reserve((size_t)n_tensors);
    for (int64_t i = 0; i < n_tensors; ++i) {
        TensorInfo t{};
        if (!c.str(&t.name)) return BH_EINVAL;
        const uint32_t nd = c.get<uint32_t>();
        if (!c.ok || nd < 1 || nd > 4) return BH_EINVAL;
        t.n_dims = (int)nd;
        int64_t ne_total = 1;
        for (int d = 0; d < 4; ++d) t.ne[d] = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            t.ne[d] = c.get<int64_t>();
            if (!c.ok || t.ne[d] < 0 || (t.ne[d] > 0 && ne_total > INT64_MAX / t.ne[d])) return BH_EINVAL;
            ne_total *= t.ne[d];
        }
        t.type = (int)c.get<int32_t>();
        t.offset = c.get<uint64_t>();
        if (!c.ok) return BH_EINVAL;
        size_t bb;
        int64_t bv;
        if (type_block(t.type, &bb, &bv)) {
            if (t.ne[0] % bv) return BH_EINVAL;
            t.bytes = (uint64_t)(ne_total / bv) * bb;
        }
        g->tensors.push_back(std::move(t));
    }
    const size_t hdr = g->size - c.left;
    g->data_off = (hdr + g->alignment - 1) / g->alignment * g->alignment;
    for (const TensorInfo& t : g->tensors) {
        if (t.offset % g->alignment) return BH_EINVAL;
        if (t.bytes && (g->data_off > g->size || t.offset > g->size - g->data_off ||
                        t.bytes > g->size - g->data_off - t.offset))
            return BH_EINVAL;  // truncated file
    }
    return BH_OK;
}

const KV* key_at(const bh_gguf* g, int64_t k) {
    return (g && k >= 0 && k < (int64_t)g->kv.size()) ? &g->kv[(size_t)k] : nullptr;
}

}  // namespace

extern "C" {

int bh_gguf_open(const char* path, bh_gguf** out) {
    if (!path || !out) return BH_EINVAL;
    *out = nullptr;
    bh_gguf* g = new bh_gguf();
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0 || st.st_size < 24) {
        bh_gguf_close(g);
        return BH_EINVAL;
    }
    g->size = (size_t)st.st_size;
    void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        g->size = 0;
        bh_gguf_close(g);
        return BH_ENOMEM;
    }
    g->map = static_cast<const uint8_t*>(m);
    const int rc = parse(g);
    if (rc != BH_OK) {
        bh_gguf_close(g);
        return rc;
    }
    *out = g;
    return BH_OK;
}

int bh_gguf_close(bh_gguf* g) {
    if (!g) return BH_EINVAL;
    if (g->map) munmap(const_cast<uint8_t*>(g->map), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return BH_OK;
}

int64_t bh_gguf_n_tensors(const bh_gguf* g) { return g ? (int64_t)g->tensors.size() : BH_EINVAL; }
int64_t bh_gguf_n_keys(const bh_gguf* g) { return g ? (int64_t)g->kv.size() : BH_EINVAL; }

int64_t bh_gguf_find_tensor(const bh_gguf* g, const char* name) {
    if (!g || !name) return -1;
    for (size_t i = 0; i < g->tensors.size(); ++i)
        if (g->tensors[i].name == name) return (int64_t)i;
    return -1;
}

int bh_gguf_tensor_info(const bh_gguf* g, int64_t i, const char** name, int* ggml_type, int* n_dims, int64_t* ne4,
                        uint64_t* file_offset, uint64_t* bytes) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return BH_EINVAL;
    const TensorInfo& t = g->tensors[(size_t)i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (ne4)
        for (int d = 0; d < 4; ++d) ne4[d] = t.ne[d];
    if (file_offset) *file_offset = g->data_off + t.offset;
    if (bytes) *bytes = t.bytes;
    return BH_OK;
}

const void* bh_gguf_tensor_host(const bh_gguf* g, int64_t i) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size() || !g->tensors[(size_t)i].bytes) return nullptr;
    return g->map + g->data_off + g->tensors[(size_t)i].offset;
}

int bh_gguf_upload(bh_ctx* ctx, const bh_gguf* g, int64_t i, void* dst, size_t dst_bytes, void* stream) {
    if (!ctx || !g || !dst || i < 0 || i >= (int64_t)g->tensors.size()) return BH_EINVAL;
    const TensorInfo& t = g->tensors[(size_t)i];
    if (!t.bytes || dst_bytes < t.bytes) return BH_EINVAL;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return BH_ENODEV;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // pageable source: the runtime stages it; the call returns once the copy is done
    if (cudaMemcpyAsync(dst, g->map + g->data_off + t.offset, t.bytes, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return BH_EIO;
    }
    return BH_OK;
}

int64_t bh_gguf_find_key(const bh_gguf* g, const char* key) {
    if (!g || !key) return -1;
    for (size_t i = 0; i < g->kv.size(); ++i)
        if (g->kv[i].key == key) return (int64_t)i;
    return -1;
}

int bh_gguf_key(const bh_gguf* g, int64_t k, const char** key, int* type) {
    const KV* kv = key_at(g, k);
    if (!kv) return BH_EINVAL;
    if (key) *key = kv->key.c_str();
    if (type) *type = (int)kv->type;
    return BH_OK;
}

int bh_gguf_get_int(const bh_gguf* g, int64_t k, int64_t* v) {
    const KV* kv = key_at(g, k);
    if (!kv || !v) return BH_EINVAL;
    switch (kv->type) {
        case GT_UINT8: { uint8_t x; std::memcpy(&x, kv->val, 1); *v = x; return BH_OK; }
        case GT_INT8: { int8_t x; std::memcpy(&x, kv->val, 1); *v = x; return BH_OK; }
        case GT_BOOL: { int8_t x; std::memcpy(&x, kv->val, 1); *v = x != 0; return BH_OK; }
        case GT_UINT16: { uint16_t x; std::memcpy(&x, kv->val, 2); *v = x; return BH_OK; }
        case GT_INT16: { int16_t x; std::memcpy(&x, kv->val, 2); *v = x; return BH_OK; }
        case GT_UINT32: { uint32_t x; std::memcpy(&x, kv->val, 4); *v = x; return BH_OK; }
        case GT_INT32: { int32_t x; std::memcpy(&x, kv->val, 4); *v = x; return BH_OK; }
        case GT_UINT64: {
            uint64_t x;
            std::memcpy(&x, kv->val, 8);
            if (x > (uint64_t)INT64_MAX) return BH_EINVAL;
            *v = (int64_t)x;
            return BH_OK;
        }
        case GT_INT64: { int64_t x; std::memcpy(&x, kv->val, 8); *v = x; return BH_OK; }
        default: return BH_EINVAL;
    }
}

int bh_gguf_get_float(const bh_gguf* g, int64_t k, double* v) {
    const KV* kv = key_at(g, k);
    if (!kv || !v) return BH_EINVAL;
    if (kv->type == GT_FLOAT32) { float x; std::memcpy(&x, kv->val, 4); *v = x; return BH_OK; }
    if (kv->type == GT_FLOAT64) { double x; std::memcpy(&x, kv->val, 8); *v = x; return BH_OK; }
    int64_t iv;
    if (bh_gguf_get_int(g, k, &iv) != BH_OK) return BH_EINVAL;
    *v = (double)iv;
    return BH_OK;
}

int bh_gguf_get_str(const bh_gguf* g, int64_t k, const char** s, uint64_t* len) {
    const KV* kv = key_at(g, k);
    if (!kv || !s || !len || kv->type != GT_STRING) return BH_EINVAL;
    uint64_t n;
    std::memcpy(&n, kv->val, 8);
    *s = reinterpret_cast<const char*>(kv->val + 8);
    *len = n;
    return BH_OK;
}

}  // extern "C"
