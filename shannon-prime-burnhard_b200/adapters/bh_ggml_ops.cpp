// bh_ggml_ops.cpp — ggml graph nodes for the reference engine's BURN_MOE
// op and the Q4_K branch of its sp_crt_mul_mat switch, computed on the B200
// through include/bh_q4k.h (see bh_ggml_ops.h for the contract).
//
// Host side only: the callbacks stage the node's inputs, call the library's
// C ABI (bh_q4k_moe / bh_q4k_moe_ep + bh_moe_combine_split for BURN_MOE,
// bh_q4k_matvec_f32 for the matmul) on the device's default stream, and
// write the node's output. Token / column counts above the library's batch of 8 run
// in chunks of 8 (every column is independent in both operations).
#include "bh_ggml_ops.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <mutex>
#include <tuple>
#include <vector>

#include "ggml-backend.h"

namespace {

constexpr int CHUNK = 8;  // the library's batch limit (BH_MAX_BATCH)

std::atomic<int> g_last_error{0};

void note_error(int rc) {
    if (rc != BH_OK) g_last_error.store(rc);
}

// Device copies of host weight tensors, keyed by (device, data, bytes).
struct WeightCache {
    std::mutex mu;
    std::map<std::tuple<int, const void*, size_t>, void*> map;
};
WeightCache& cache() {
    static WeightCache c;
    return c;
}

bool host_tensor(const ggml_tensor* t) { return t->buffer == nullptr || ggml_backend_buffer_is_host(t->buffer); }

// The device address of a weight tensor: in place when it lives in device
// memory, else a cached upload of its bytes.
const void* device_weights(bh_ctx* ctx, int device, const ggml_tensor* t) {
    if (!t || !t->data) return nullptr;
    const size_t bytes = ggml_nbytes(t);
    if (!host_tensor(t)) return t->data;  // a backend buffer on the GPU
    WeightCache& c = cache();
    std::lock_guard<std::mutex> lock(c.mu);
    const auto key = std::make_tuple(device, static_cast<const void*>(t->data), bytes);
    auto it = c.map.find(key);
    if (it != c.map.end()) return it->second;
    (void)ctx;
    void* d = nullptr;  // (one upload per weight tensor and device)
    if (cudaSetDevice(device) != cudaSuccess || cudaMalloc(&d, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaMemcpy(d, t->data, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return nullptr;
    }
    c.map[key] = d;
    return d;
}

// Bytes [off, off + size) of a tensor into host memory.
void read_tensor(const ggml_tensor* t, void* dst, size_t off, size_t size) {
    if (host_tensor(t))
        std::memcpy(dst, static_cast<const char*>(t->data) + off, size);
    else
        ggml_backend_tensor_get(t, dst, off, size);
}

void write_tensor(ggml_tensor* t, const void* src, size_t off, size_t size) {
    if (host_tensor(t))
        std::memcpy(static_cast<char*>(t->data) + off, src, size);
    else
        ggml_backend_tensor_set(t, src, off, size);
}

struct Device {
    int id = -1;
};

// The context's device, made current for the staging copies here.
bool ctx_device(bh_ctx* ctx, Device& d) {
    d.id = bh_ctx_device(ctx);
    return d.id >= 0 && cudaSetDevice(d.id) == cudaSuccess;
}

// Node user data outlives the graph that holds the node (a graph may be
// recomputed many times); it is kept here until bh_ggml_ops_release.
std::mutex g_user_mu;
std::vector<void*> g_user;

template <class T>
T* new_user() {
    T* u = new (std::nothrow) T();
    if (!u) return nullptr;
    std::lock_guard<std::mutex> lock(g_user_mu);
    g_user.push_back(u);
    return u;
}

// ---------------------------------------------------------------------------
// BURN_MOE
// ---------------------------------------------------------------------------
struct MoeUser {
    bh_ctx* ctx;
    int k;
    int pivot;  // experts [0, pivot) in the *_cpu banks; 0: one bank
    const ggml_tensor* gate_cpu;
    const ggml_tensor* up_cpu;
    const ggml_tensor* down_cpu;
};

void burn_moe_compute(ggml_tensor* dst, int ith, int nth, void* userdata) {
    (void)nth;
    if (ith != 0) return;
    const MoeUser* u = static_cast<const MoeUser*>(userdata);
    const ggml_tensor* cur = dst->src[0];
    const ggml_tensor* sel = dst->src[1];
    const ggml_tensor* wts = dst->src[2];
    const ggml_tensor* gate = dst->src[3];
    const ggml_tensor* up = dst->src[4];
    const ggml_tensor* down = dst->src[5];
    const int n_embd = (int)cur->ne[0], n_tok = (int)cur->ne[1], k = u->k;
    const int n_ff = (int)gate->ne[1];
    const int n_expert = u->pivot + (int)gate->ne[2];
    std::vector<float> out((size_t)n_embd * n_tok, 0.f);
    int rc = BH_OK;
    if (cur->type != GGML_TYPE_F32 || sel->type != GGML_TYPE_I32 || wts->type != GGML_TYPE_F32 ||
        gate->type != GGML_TYPE_Q4_K || up->type != GGML_TYPE_Q4_K || down->type != GGML_TYPE_Q4_K ||
        !ggml_is_contiguous(cur) || !ggml_is_contiguous(sel) || !ggml_is_contiguous(wts) || sel->ne[0] != k ||
        (int)down->ne[1] != n_embd)
        rc = BH_EINVAL;
    Device dv;
    if (rc == BH_OK && !ctx_device(u->ctx, dv)) rc = BH_ENODEV;
    const void *g = nullptr, *uu = nullptr, *dd = nullptr, *gc = nullptr, *uc = nullptr, *dc = nullptr;
    if (rc == BH_OK) {
        g = device_weights(u->ctx, dv.id, gate);
        uu = device_weights(u->ctx, dv.id, up);
        dd = device_weights(u->ctx, dv.id, down);
        if (u->pivot > 0) {
            gc = device_weights(u->ctx, dv.id, u->gate_cpu);
            uc = device_weights(u->ctx, dv.id, u->up_cpu);
            dc = device_weights(u->ctx, dv.id, u->down_cpu);
        }
        if (!g || !uu || !dd || (u->pivot > 0 && (!gc || !uc || !dc))) rc = BH_ENOMEM;
    }
    // device staging for one chunk of tokens
    float *d_cur = nullptr, *d_w = nullptr, *d_out = nullptr, *d_da = nullptr, *d_db = nullptr;
    int32_t* d_sel = nullptr;
    const size_t pairs = (size_t)CHUNK * k;
    if (rc == BH_OK &&
        (cudaMalloc(&d_cur, sizeof(float) * CHUNK * n_embd) != cudaSuccess ||
         cudaMalloc(&d_w, sizeof(float) * pairs) != cudaSuccess ||
         cudaMalloc(&d_sel, sizeof(int32_t) * pairs) != cudaSuccess ||
         cudaMalloc(&d_out, sizeof(float) * CHUNK * n_embd) != cudaSuccess ||
         (u->pivot > 0 && (cudaMalloc(&d_da, sizeof(float) * pairs * n_embd) != cudaSuccess ||
                           cudaMalloc(&d_db, sizeof(float) * pairs * n_embd) != cudaSuccess))))
        rc = BH_ENOMEM;
    std::vector<float> hcur((size_t)CHUNK * n_embd), hw(pairs);
    std::vector<int32_t> hsel(pairs);
    for (int t0 = 0; t0 < n_tok && rc == BH_OK; t0 += CHUNK) {
        const int nt = n_tok - t0 < CHUNK ? n_tok - t0 : CHUNK;
        read_tensor(cur, hcur.data(), sizeof(float) * (size_t)t0 * n_embd, sizeof(float) * (size_t)nt * n_embd);
        read_tensor(sel, hsel.data(), sizeof(int32_t) * (size_t)t0 * k, sizeof(int32_t) * (size_t)nt * k);
        read_tensor(wts, hw.data(), sizeof(float) * (size_t)t0 * k, sizeof(float) * (size_t)nt * k);
        if (cudaMemcpy(d_cur, hcur.data(), sizeof(float) * (size_t)nt * n_embd, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d_sel, hsel.data(), sizeof(int32_t) * (size_t)nt * k, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d_w, hw.data(), sizeof(float) * (size_t)nt * k, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = BH_EIO;
            break;
        }
        if (u->pivot == 0) {
            rc = bh_q4k_moe(u->ctx, d_cur, nt, d_sel, d_w, nullptr, 0, g, uu, dd, n_expert, n_embd, n_ff, k, d_out,
                            nullptr, nullptr, BH_FOLD_X86, nullptr);
        } else {
            // the two sub-banks as two expert-parallel shares on this device
            rc = bh_q4k_moe_ep(u->ctx, d_cur, nt, d_sel, d_w, nullptr, 0, gc, uc, dc, n_expert, 0, u->pivot, n_embd,
                               n_ff, k, d_da, nullptr, nullptr, BH_FOLD_X86, nullptr);
            if (rc == BH_OK)
                rc = bh_q4k_moe_ep(u->ctx, d_cur, nt, d_sel, d_w, nullptr, 0, g, uu, dd, n_expert, u->pivot, n_expert,
                                   n_embd, n_ff, k, d_db, nullptr, nullptr, BH_FOLD_X86, nullptr);
            if (rc == BH_OK) rc = bh_moe_combine_split(u->ctx, d_da, d_db, d_w, nt, k, n_embd, d_out, 0, nullptr);
        }
        if (rc == BH_OK && cudaMemcpy(out.data() + (size_t)t0 * n_embd, d_out, sizeof(float) * (size_t)nt * n_embd,
                                      cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = BH_EIO;
        if (rc == BH_OK) rc = bh_device_status(u->ctx, 1);
    }
    cudaFree(d_cur);
    cudaFree(d_w);
    cudaFree(d_sel);
    cudaFree(d_out);
    cudaFree(d_da);
    cudaFree(d_db);
    note_error(rc);
    write_tensor(dst, out.data(), 0, sizeof(float) * out.size());
}

// ---------------------------------------------------------------------------
// Q4_K matmul
// ---------------------------------------------------------------------------
void mul_mat_compute(ggml_tensor* dst, int ith, int nth, void* userdata) {
    (void)nth;
    if (ith != 0) return;
    bh_ctx* ctx = static_cast<bh_ctx*>(userdata);
    const ggml_tensor* W = dst->src[0];
    const ggml_tensor* x = dst->src[1];
    const int64_t K = W->ne[0], M = W->ne[1], N = x->ne[1];
    std::vector<float> y((size_t)M * N, 0.f);
    int rc = BH_OK;
    if (W->type != GGML_TYPE_Q4_K || x->type != GGML_TYPE_F32 || x->ne[0] != K || !ggml_is_contiguous(x) ||
        x->ne[2] != 1 || x->ne[3] != 1)
        rc = BH_EINVAL;
    Device dv;
    if (rc == BH_OK && !ctx_device(ctx, dv)) rc = BH_ENODEV;
    const void* w = rc == BH_OK ? device_weights(ctx, dv.id, W) : nullptr;
    if (rc == BH_OK && !w) rc = BH_ENOMEM;
    float *d_x = nullptr, *d_y = nullptr;
    if (rc == BH_OK && (cudaMalloc(&d_x, sizeof(float) * CHUNK * K) != cudaSuccess ||
                        cudaMalloc(&d_y, sizeof(float) * CHUNK * M) != cudaSuccess))
        rc = BH_ENOMEM;
    std::vector<float> hx((size_t)CHUNK * K);
    for (int64_t n0 = 0; n0 < N && rc == BH_OK; n0 += CHUNK) {
        const int nb = (int)(N - n0 < CHUNK ? N - n0 : CHUNK);
        read_tensor(x, hx.data(), sizeof(float) * (size_t)(n0 * K), sizeof(float) * (size_t)nb * K);
        if (cudaMemcpy(d_x, hx.data(), sizeof(float) * (size_t)nb * K, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = BH_EIO;
            break;
        }
        // y[b][m] = W[m] . x[b]: ggml_mul_mat's dst [M, N]
        rc = bh_q4k_matvec_f32(ctx, w, M, K, d_x, nb, d_y, BH_FOLD_X86, nullptr);
        if (rc == BH_OK && cudaMemcpy(y.data() + (size_t)(n0 * M), d_y, sizeof(float) * (size_t)nb * M,
                                      cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = BH_EIO;
        if (rc == BH_OK) rc = bh_device_status(ctx, 1);
    }
    cudaFree(d_x);
    cudaFree(d_y);
    note_error(rc);
    write_tensor(dst, y.data(), 0, sizeof(float) * y.size());
}

}  // namespace

extern "C" {

ggml_tensor* bh_build_burn_moe_op(ggml_context* gctx, ggml_tensor* cur, ggml_tensor* selected, ggml_tensor* weights,
                                  ggml_tensor* gate_exps, ggml_tensor* up_exps, ggml_tensor* down_exps,
                                  ggml_tensor* gate_exps_cpu, ggml_tensor* up_exps_cpu, ggml_tensor* down_exps_cpu,
                                  int n_expert_used, int pivot, bh_ctx* ctx) {
    if (!gctx || !cur || !selected || !weights || !gate_exps || !up_exps || !down_exps || !ctx || n_expert_used < 1)
        return nullptr;
    MoeUser* u = new_user<MoeUser>();
    if (!u) return nullptr;
    u->ctx = ctx;
    u->k = n_expert_used;
    const bool split = gate_exps_cpu && up_exps_cpu && down_exps_cpu && pivot > 0;
    u->pivot = split ? pivot : 0;
    u->gate_cpu = split ? gate_exps_cpu : nullptr;
    u->up_cpu = split ? up_exps_cpu : nullptr;
    u->down_cpu = split ? down_exps_cpu : nullptr;
    ggml_tensor* args[6] = {cur, selected, weights, gate_exps, up_exps, down_exps};
    return ggml_custom_4d(gctx, GGML_TYPE_F32, cur->ne[0], cur->ne[1], 1, 1, args, 6, burn_moe_compute, 1, u);
}

ggml_tensor* bh_ggml_mul_mat(ggml_context* gctx, ggml_tensor* W, ggml_tensor* x, bh_ctx* ctx) {
    if (!gctx || !W || !x) return nullptr;
    if (!ctx || W->type != GGML_TYPE_Q4_K || x->type != GGML_TYPE_F32) return ggml_mul_mat(gctx, W, x);
    ggml_tensor* args[2] = {W, x};
    return ggml_custom_4d(gctx, GGML_TYPE_F32, W->ne[1], x->ne[1], 1, 1, args, 2, mul_mat_compute, 1, ctx);
}

int bh_ggml_ops_last_error(void) { return g_last_error.exchange(0); }

int bh_ggml_ops_cached_weights(void) {
    WeightCache& c = cache();
    std::lock_guard<std::mutex> lock(c.mu);
    return (int)c.map.size();
}

void bh_ggml_ops_release(void) {
    WeightCache& c = cache();
    {
        std::lock_guard<std::mutex> lock(c.mu);
        for (auto& kv : c.map) {
            cudaSetDevice(std::get<0>(kv.first));
            cudaFree(kv.second);
        }
        c.map.clear();
    }
    std::lock_guard<std::mutex> lock(g_user_mu);
    for (void* u : g_user) delete static_cast<MoeUser*>(u);
    g_user.clear();
}

}  // extern "C"
