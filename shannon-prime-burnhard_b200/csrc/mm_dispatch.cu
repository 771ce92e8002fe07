// mm_dispatch.cu — the native engine's dense-matmul hook served by the Q4_K
// kernels.
//
// The reference's native forward (desktop/engine/src/forward_native.cpp
// weight_matmul, :102-118) calls layer.mm_dispatch(userdata, lhs [M][K] fp32,
// W_fp16 [K][N], M, K, N, out [M][N] fp32) first and falls back to its CPU
// matmul when the hook returns non-zero (forward_native.h:115-119). The hook
// receives the fp16 copy of a weight, which is only a key here: the engine
// registers, at bind time, the device Q4_K bytes of the same weight (its GGUF
// rows, N x K) under that key, and bh_mm_dispatch computes out[m][n] =
// W_q4k[n] . lhs[m] with lhs quantized to Q8_K, as ggml's own Q4_K matmul
// does (not the fp32 dequantized product of the CPU fallback). Unregistered
// keys and shapes that do not match the registration return non-zero, so
// the engine falls through exactly as with no hook.
#include <mutex>
#include <new>
#include <unordered_map>

#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

struct bh_mm_registry {
    bh_ctx* ctx = nullptr;
    std::mutex mu;
    struct Entry {
        const void* w;
        int n, k;
    };
    std::unordered_map<const void*, Entry> map;
};

extern "C" {

int bh_mm_registry_create(bh_ctx* ctx, bh_mm_registry** out) {
    if (!ctx || !out) return BH_EINVAL;
    bh_mm_registry* r = new (std::nothrow) bh_mm_registry();
    if (!r) return BH_ENOMEM;
    r->ctx = ctx;
    *out = r;
    return BH_OK;
}

int bh_mm_registry_add(bh_mm_registry* r, const void* key, const void* W_q4k, int N, int K) {
    if (!r || !key || !W_q4k || N < 1 || K < bh::QK || K % bh::QK) return BH_EINVAL;
    if (reinterpret_cast<uintptr_t>(W_q4k) % 16) return BH_EINVAL;
    std::lock_guard<std::mutex> lock(r->mu);
    r->map[key] = bh_mm_registry::Entry{W_q4k, N, K};
    return BH_OK;
}

int bh_mm_registry_free(bh_mm_registry* r) {
    if (!r) return BH_EINVAL;
    delete r;
    return BH_OK;
}

int bh_mm_dispatch(void* userdata, const float* lhs, const uint16_t* W_fp16, int M, int K, int N, float* out) {
    bh_mm_registry* r = static_cast<bh_mm_registry*>(userdata);
    if (!r || !lhs || !W_fp16 || !out || M < 1) return BH_EINVAL;
    bh_mm_registry::Entry e;
    {
        std::lock_guard<std::mutex> lock(r->mu);
        auto it = r->map.find(static_cast<const void*>(W_fp16));
        if (it == r->map.end()) return BH_EINVAL;  // not ours: the engine falls through
        e = it->second;
    }
    if (e.k != K || e.n != N) return BH_EINVAL;
    // rows of lhs are the columns of the matvec, BH_MAX_BATCH at a time
    for (int m0 = 0; m0 < M; m0 += BH_MAX_BATCH) {
        const int b = M - m0 < BH_MAX_BATCH ? M - m0 : BH_MAX_BATCH;
        const int rc = bh_q4k_mul_mat_host(r->ctx, e.w, N, K, lhs + (size_t)m0 * K, b, out + (size_t)m0 * N,
                                           BH_FOLD_X86);
        if (rc != BH_OK) return rc;
    }
    return BH_OK;
}

}  // extern "C"
