// moe_api.cu — the routed-expert FFN entry points (bh_moe_route,
// bh_q4k_moe) and the 30B-A3B-shaped MoE layer stack.
//
// Host-side argument checks happen before any launch; an invalid call
// launches nothing and returns BH_EINVAL. An out-of-range or repeated expert
// id in a given routing is caught on the device: the kernel skips all work
// and sets the device status (bh_device_status returns BH_EINVAL).
#include <cstring>
#include <vector>

#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace {

struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool moe_shape_ok(int n_tok, int n_expert, int n_embd, int n_ff, int k) {
    return n_tok >= 1 && n_tok <= bh::MOE_MAX_TOK && k >= 1 && k <= bh::MOE_MAX_K && n_expert >= k &&
           n_expert <= bh::MOE_MAX_EXPERT && n_embd >= bh::QK && n_embd % bh::QK == 0 &&
           n_embd <= bh::QK * bh::MOE_MAX_EMBD_BLOCKS && n_ff >= bh::QK &&
           n_ff % bh::QK == 0 && (int64_t)n_expert * n_ff < ((int64_t)1 << 31) &&
           (int64_t)n_expert * n_embd < ((int64_t)1 << 31);
}

int ensure_moe_scratch(bh_ctx* ctx, size_t bytes) {
    if (ctx->moe_scratch_bytes >= bytes) return BH_OK;
    if (ctx->moe_scratch) {
        cudaDeviceSynchronize();
        bh::unregister_barrier_words(ctx, ctx->moe_scratch);
        cudaFree(ctx->moe_scratch);
        ctx->moe_scratch = nullptr;
        ctx->moe_scratch_bytes = 0;
    }
    if (cudaMalloc(&ctx->moe_scratch, bytes) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    // the grid-barrier words live in the first 256 bytes and must start at zero
    if (cudaMemset(ctx->moe_scratch, 0, 256) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(ctx->moe_scratch);
        ctx->moe_scratch = nullptr;
        return BH_EIO;
    }
    ctx->moe_scratch_bytes = bytes;
    bh::register_barrier_words(ctx, ctx->moe_scratch);
    return BH_OK;
}

bh::MoeParams moe_base(bh_ctx* ctx, int n_tok, int n_expert, int n_embd, int n_ff, int k) {
    bh::MoeParams p;
    std::memset(&p, 0, sizeof(p));
    p.n_expert = n_expert;
    p.n_embd = n_embd;
    p.n_ff = n_ff;
    p.k = k;
    p.B = n_tok;
    p.n_layer = 1;
    p.e_lo = 0;
    p.e_hi = n_expert;
    p.combine = 1;
    p.gbar_wait = ctx->barrier_wait_cycles;
    p.status = ctx->d_status;
#ifdef BH_TRACE
    p.trace = ctx->trace;
#endif
    return p;
}

}  // namespace

namespace bh {

// One CTA per SM with the whole shared memory: the ring then holds enough
// slots that at batch 1 every warp's gate|up and down rows are in flight at
// once.
int run_moe(bh_ctx* ctx, MoeParams& p, int fold, cudaStream_t s, bool pdl) {
    int rc = moe_plan(p, 200 * 1024, ctx->moe_stage_bytes);
    if (rc != BH_OK) return rc;
    LaunchOpts o;
    o.stream = s;
    o.pdl = pdl;
    o.grid = ctx->num_sms;
    return launch_moe(p, fold, o);
}

}  // namespace bh

extern "C" {

int bh_moe_route(bh_ctx* ctx, const float* logits, int n_tok, int n_expert, int k, int norm_topk,
                 int32_t* selected_out, float* weights_out, void* stream) {
    if (!ctx || !logits || !selected_out || !weights_out) return BH_EINVAL;
    if (n_tok < 1 || n_tok > bh::MOE_MAX_TOK || k < 1 || k > bh::MOE_MAX_K || n_expert < k ||
        n_expert > bh::MOE_MAX_EXPERT)
        return BH_EINVAL;
    if (!aligned(logits, 4) || !aligned(selected_out, 4) || !aligned(weights_out, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    bh::MoeParams p = moe_base(ctx, n_tok, n_expert, bh::QK, bh::QK, k);
    p.norm_topk = norm_topk ? 1 : 0;
    p.logits = logits;
    p.ids_out = selected_out;
    p.w_out = weights_out;
    bh::LaunchOpts o;
    o.stream = static_cast<cudaStream_t>(stream);
    return bh::launch_moe_route(p, o);
}

int bh_q4k_moe(bh_ctx* ctx, const float* cur, int n_tok, const int32_t* selected, const float* weights,
               const float* router_logits, int norm_topk, const void* gate_exps, const void* up_exps,
               const void* down_exps, int n_expert, int n_embd, int n_ff, int k, float* out,
               int32_t* selected_out, float* weights_out, int fold, void* stream) {
    if (!ctx || !cur || !out || !gate_exps || !up_exps || !down_exps) return BH_EINVAL;
    if (!moe_shape_ok(n_tok, n_expert, n_embd, n_ff, k)) return BH_EINVAL;
    if (fold != BH_FOLD_X86 && fold != BH_FOLD_GENERIC) return BH_EINVAL;
    const bool given = selected || weights;
    if (given && (!selected || !weights || router_logits)) return BH_EINVAL;
    if (!given && !router_logits) return BH_EINVAL;
    if (!aligned(cur, 16) || !aligned(out, 4) || !aligned(gate_exps, 16) || !aligned(up_exps, 16) ||
        !aligned(down_exps, 16))
        return BH_EINVAL;
    if ((selected && !aligned(selected, 4)) || (weights && !aligned(weights, 4)) ||
        (router_logits && !aligned(router_logits, 4)) || (selected_out && !aligned(selected_out, 4)) ||
        (weights_out && !aligned(weights_out, 4)))
        return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    // scratch: barrier words (256 bytes), gate|up [n_tok*k][2*n_ff],
    // outputs [n_tok*k][n_embd], routing [n_tok*k] x 2
    const size_t pairs = (size_t)n_tok * k;
    const size_t gu_f = pairs * 2 * n_ff, do_f = pairs * n_embd;
    const size_t bytes = 256 + (gu_f + do_f + 2 * pairs) * sizeof(float);
    int rc = ensure_moe_scratch(ctx, bytes);
    if (rc != BH_OK) return rc;
    bh::MoeParams p = moe_base(ctx, n_tok, n_expert, n_embd, n_ff, k);
    p.w[0] = static_cast<const uint8_t*>(gate_exps);
    p.w[1] = static_cast<const uint8_t*>(up_exps);
    p.w[2] = static_cast<const uint8_t*>(down_exps);
    p.norm_topk = norm_topk ? 1 : 0;
    p.h = cur;
    p.gbar = reinterpret_cast<unsigned int*>(ctx->moe_scratch);
    p.gu = reinterpret_cast<float*>(ctx->moe_scratch + 256);
    p.dout = p.gu + gu_f;
    p.out = out;
    p.residual = 0;
    if (given) {
        p.ids_in = selected;
        p.w_in = weights;
    } else {
        p.logits = router_logits;
        p.ids_out = selected_out ? selected_out : reinterpret_cast<int32_t*>(p.dout + do_f);
        p.w_out = weights_out ? weights_out : p.dout + do_f + pairs;
    }
    return bh::run_moe(ctx, p, fold, static_cast<cudaStream_t>(stream), false);
}

int bh_q4k_moe_ep(bh_ctx* ctx, const float* cur, int n_tok, const int32_t* selected, const float* weights,
                  const float* router_logits, int norm_topk, const void* gate_own, const void* up_own,
                  const void* down_own, int n_expert, int expert_lo, int expert_hi, int n_embd, int n_ff, int k,
                  float* dout, int32_t* selected_out, float* weights_out, int fold, void* stream) {
    if (!ctx || !cur || !dout || !gate_own || !up_own || !down_own) return BH_EINVAL;
    if (!moe_shape_ok(n_tok, n_expert, n_embd, n_ff, k)) return BH_EINVAL;
    if (expert_lo < 0 || expert_hi > n_expert || expert_lo >= expert_hi) return BH_EINVAL;
    if (fold != BH_FOLD_X86 && fold != BH_FOLD_GENERIC) return BH_EINVAL;
    const bool given = selected || weights;
    if (given && (!selected || !weights || router_logits)) return BH_EINVAL;
    if (!given && !router_logits) return BH_EINVAL;
    if (!aligned(cur, 16) || !aligned(dout, 4) || !aligned(gate_own, 16) || !aligned(up_own, 16) ||
        !aligned(down_own, 16))
        return BH_EINVAL;
    if ((selected && !aligned(selected, 4)) || (weights && !aligned(weights, 4)) ||
        (router_logits && !aligned(router_logits, 4)) || (selected_out && !aligned(selected_out, 4)) ||
        (weights_out && !aligned(weights_out, 4)))
        return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    const size_t pairs = (size_t)n_tok * k;
    const size_t gu_f = pairs * 2 * n_ff;
    const size_t bytes = 256 + (gu_f + 2 * pairs) * sizeof(float);
    int rc = ensure_moe_scratch(ctx, bytes);
    if (rc != BH_OK) return rc;
    bh::MoeParams p = moe_base(ctx, n_tok, n_expert, n_embd, n_ff, k);
    p.w[0] = static_cast<const uint8_t*>(gate_own);
    p.w[1] = static_cast<const uint8_t*>(up_own);
    p.w[2] = static_cast<const uint8_t*>(down_own);
    p.e_lo = expert_lo;
    p.e_hi = expert_hi;
    p.combine = 0;
    p.norm_topk = norm_topk ? 1 : 0;
    p.h = cur;
    p.gbar = reinterpret_cast<unsigned int*>(ctx->moe_scratch);
    p.gu = reinterpret_cast<float*>(ctx->moe_scratch + 256);
    p.dout = dout;
    if (given) {
        p.ids_in = selected;
        p.w_in = weights;
    } else {
        p.logits = router_logits;
        p.ids_out = selected_out ? selected_out : reinterpret_cast<int32_t*>(p.gu + gu_f);
        p.w_out = weights_out ? weights_out : p.gu + gu_f + pairs;
    }
    return bh::run_moe(ctx, p, fold, static_cast<cudaStream_t>(stream), false);
}

int bh_moe_combine(bh_ctx* ctx, const float* dout, const float* weights, int n_tok, int k, int n_embd, float* out,
                   int residual, void* stream) {
    if (!ctx || !dout || !weights || !out || n_tok < 1 || n_tok > bh::MOE_MAX_TOK || k < 1 || k > bh::MOE_MAX_K ||
        n_embd < 1)
        return BH_EINVAL;
    if (!aligned(dout, 4) || !aligned(weights, 4) || !aligned(out, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    bh::LaunchOpts o;
    o.stream = static_cast<cudaStream_t>(stream);
    return bh::launch_moe_combine(dout, weights, n_tok, k, n_embd, out, residual != 0, o);
}

int bh_moe_combine_split(bh_ctx* ctx, const float* dout_a, const float* dout_b, const float* weights, int n_tok, int k,
                         int n_embd, float* out, int residual, void* stream) {
    if (!ctx || !dout_a || !dout_b || !weights || !out || n_tok < 1 || n_tok > bh::MOE_MAX_TOK || k < 1 ||
        k > bh::MOE_MAX_K || n_embd < 1)
        return BH_EINVAL;
    if (!aligned(dout_a, 4) || !aligned(dout_b, 4) || !aligned(weights, 4) || !aligned(out, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    bh::LaunchOpts o;
    o.stream = static_cast<cudaStream_t>(stream);
    return bh::launch_moe_combine(dout_a, weights, n_tok, k, n_embd, out, residual != 0, o, dout_b);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// the MoE layer stack
// ---------------------------------------------------------------------------
struct bh_moe_stack {
    bh_ctx* ctx = nullptr;
    bh_moe_config cfg{};
    cudaStream_t stream = nullptr;
    uint8_t* wbuf = nullptr;    // gate banks of all layers, then up banks, then down banks
    size_t gate_bytes = 0;      // one gate (or up) bank
    size_t down_bytes = 0;      // one down bank
    float* fbuf = nullptr;      // logits, norm, h, gu, dout, weights
    float* logits = nullptr;    // [L][T][E]
    float* norm = nullptr;      // [L][n_embd]
    float* h = nullptr;         // [T][n_embd]
    float* gu = nullptr;        // [T*k][2*n_ff]
    float* dout = nullptr;      // [T*k][n_embd]
    float* wsel = nullptr;      // [L][T][k]
    int32_t* ids = nullptr;     // [L][T][k]
    unsigned int* gbar = nullptr;  // grid-barrier words of the layer kernels
    float* host_h = nullptr;    // pinned [T][n_embd]
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

uint64_t moe_tensor_seed(uint64_t seed, int layer, int which) {
    uint64_t z = seed ^ (0x3c6ef372fe94f82bULL + (uint64_t)(layer + 1) * 0x9e3779b97f4a7c15ULL +
                         (uint64_t)which * 0xd6e8feb86659fd93ULL);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

const uint8_t* layer_bank(const bh_moe_stack* st, int l, int which) {
    const size_t L = (size_t)st->cfg.n_layer;
    if (which == BH_MOE_DOWN) return st->wbuf + 2 * L * st->gate_bytes + (size_t)l * st->down_bytes;
    return st->wbuf + ((size_t)which * L + (size_t)l) * st->gate_bytes;
}

// One cooperative launch per layer (a single launch looping over all layers
// measured slower: its extra grid barrier per layer costs more than the
// programmatic-launch boundary it replaces).
int enqueue_moe_step(bh_moe_stack* st, cudaStream_t s) {
    const bh_moe_config& c = st->cfg;
    for (int l = 0; l < c.n_layer; ++l) {
        bh::MoeParams p = moe_base(st->ctx, c.n_tok, c.n_expert, c.n_embd, c.n_ff, c.k);
        p.w[0] = layer_bank(st, l, BH_MOE_GATE);
        p.w[1] = layer_bank(st, l, BH_MOE_UP);
        p.w[2] = layer_bank(st, l, BH_MOE_DOWN);
        p.norm_topk = 1;
        p.logits = st->logits + (size_t)l * c.n_tok * c.n_expert;
        p.ids_out = st->ids + (size_t)l * c.n_tok * c.k;
        p.w_out = st->wsel + (size_t)l * c.n_tok * c.k;
        p.h = st->h;
        p.gamma = st->norm + (size_t)l * c.n_embd;
        p.eps = c.rms_eps;
        p.gu = st->gu;
        p.dout = st->dout;
        p.out = st->h;
        p.residual = 1;
        p.gbar = st->gbar;
        const int rc = bh::run_moe(st->ctx, p, BH_FOLD_X86, s, true);
        if (rc != BH_OK) return rc;
    }
    return BH_OK;
}

int ensure_moe_graph(bh_moe_stack* st) {
    if (st->exec) return BH_OK;
    if (cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return BH_EIO;
    const int rc = enqueue_moe_step(st, st->stream);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(st->stream, &g);
    if (rc != BH_OK || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc != BH_OK ? rc : BH_EIO;
    }
    if (cudaGraphInstantiate(&st->exec, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        cudaGetLastError();
        return BH_EIO;
    }
    st->graph = g;
    return BH_OK;
}

}  // namespace

extern "C" {

void bh_moe_default_config(bh_moe_config* cfg) {
    if (!cfg) return;
    cfg->n_layer = 48;
    cfg->n_embd = 2048;
    cfg->n_ff = 768;
    cfg->n_expert = 128;
    cfg->k = 8;
    cfg->n_tok = 1;
    cfg->rms_eps = 1e-6f;
}

int bh_moe_stack_free(bh_moe_stack* st) {
    if (!st) return BH_EINVAL;
    DeviceGuard g(st->ctx->device);
    if (st->stream) cudaStreamSynchronize(st->stream);
    if (st->exec) cudaGraphExecDestroy(st->exec);
    if (st->graph) cudaGraphDestroy(st->graph);
    if (st->wbuf) cudaFree(st->wbuf);
    if (st->fbuf) cudaFree(st->fbuf);
    if (st->ids) cudaFree(st->ids);
    if (st->gbar) {
        bh::unregister_barrier_words(st->ctx, st->gbar);
        cudaFree(st->gbar);
    }
    if (st->host_h) cudaFreeHost(st->host_h);
    if (st->stream) cudaStreamDestroy(st->stream);
    delete st;
    return BH_OK;
}

int bh_moe_stack_create(bh_ctx* ctx, const bh_moe_config* cfg, uint64_t seed, bh_moe_stack** out) {
    if (!ctx || !cfg || !out) return BH_EINVAL;
    const bh_moe_config c = *cfg;
    if (c.n_layer < 1 || !moe_shape_ok(c.n_tok, c.n_expert, c.n_embd, c.n_ff, c.k) || !(c.rms_eps > 0.f))
        return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return BH_ENODEV;
    bh_moe_stack* st = new bh_moe_stack;
    st->ctx = ctx;
    st->cfg = c;
    st->gate_bytes = (size_t)c.n_expert * c.n_ff * (c.n_embd / bh::QK) * bh::Q4K_BYTES;
    st->down_bytes = (size_t)c.n_expert * c.n_embd * (c.n_ff / bh::QK) * bh::Q4K_BYTES;
    const size_t wtotal = (size_t)c.n_layer * (2 * st->gate_bytes + st->down_bytes);
    const size_t pairs = (size_t)c.n_tok * c.k;
    const size_t n_logit = (size_t)c.n_layer * c.n_tok * c.n_expert, n_norm = (size_t)c.n_layer * c.n_embd;
    const size_t n_h = (size_t)c.n_tok * c.n_embd, n_gu = pairs * 2 * c.n_ff, n_do = pairs * c.n_embd;
    const size_t n_w = (size_t)c.n_layer * pairs;
    auto up4 = [](size_t n) { return (n + 3) & ~(size_t)3; };  // keep every array 16-byte aligned
    const size_t ftotal = up4(n_logit) + up4(n_norm) + up4(n_h) + up4(n_gu) + up4(n_do) + up4(n_w);
    if (cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&st->wbuf, wtotal) != cudaSuccess || cudaMalloc(&st->fbuf, ftotal * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&st->ids, n_w * sizeof(int32_t)) != cudaSuccess || cudaMalloc(&st->gbar, 256) != cudaSuccess ||
        cudaMemset(st->gbar, 0, 256) != cudaSuccess ||
        cudaMallocHost(&st->host_h, n_h * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        bh_moe_stack_free(st);
        return BH_ENOMEM;
    }
    bh::register_barrier_words(ctx, st->gbar);
    float* f = st->fbuf;
    st->logits = f; f += up4(n_logit);
    st->norm = f; f += up4(n_norm);
    st->h = f; f += up4(n_h);
    st->gu = f; f += up4(n_gu);
    st->dout = f; f += up4(n_do);
    st->wsel = f;
    int rc = BH_OK;
    if ((rc = bh::fill_normal(st->logits, (int64_t)n_logit, 0, moe_tensor_seed(seed, -1, 1), 0.0, 1.0, st->stream)) ||
        (rc = bh::fill_normal(st->norm, (int64_t)n_norm, 0, moe_tensor_seed(seed, -1, 2), 1.0, 0.02, st->stream)) ||
        (rc = bh::fill_normal(st->h, (int64_t)n_h, 0, moe_tensor_seed(seed, -1, 3), 0.0, 1.0, st->stream))) {
        bh_moe_stack_free(st);
        return rc;
    }
    // expert banks: seeded N(0, 0.02) in fp32 chunks, quantized on the device
    const size_t chunk_floats = (size_t)64 << 20;
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, chunk_floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        bh_moe_stack_free(st);
        return BH_ENOMEM;
    }
    for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) {
        for (int which = 0; which < 3 && rc == BH_OK; ++which) {
            const int64_t rows = (int64_t)c.n_expert * (which == BH_MOE_DOWN ? c.n_embd : c.n_ff);
            const int64_t k = which == BH_MOE_DOWN ? c.n_ff : c.n_embd;
            const int64_t rows_per_chunk = (int64_t)(chunk_floats / (size_t)k);
            const uint64_t ts = moe_tensor_seed(seed, l, 10 + which);
            uint8_t* dst = const_cast<uint8_t*>(layer_bank(st, l, which));
            for (int64_t r0 = 0; r0 < rows && rc == BH_OK; r0 += rows_per_chunk) {
                const int64_t nr = rows - r0 < rows_per_chunk ? rows - r0 : rows_per_chunk;
                rc = bh::fill_normal(tmp, nr * k, r0 * k, ts, 0.0, 0.02, st->stream);
                if (rc == BH_OK)
                    rc = bh::launch_q4k_quantize(tmp, nr, k, dst + (size_t)r0 * (k / bh::QK) * bh::Q4K_BYTES,
                                                 st->stream);
            }
        }
    }
    cudaStreamSynchronize(st->stream);
    cudaFree(tmp);
    if (rc != BH_OK || cudaGetLastError() != cudaSuccess) {
        bh_moe_stack_free(st);
        return rc != BH_OK ? rc : BH_EIO;
    }
    *out = st;
    return BH_OK;
}

int bh_moe_stack_step(bh_moe_stack* st, const float* h, float* h_out, void* stream) {
    if (!st || !h || !h_out || !aligned(h, 4) || !aligned(h_out, 4)) return BH_EINVAL;
    DeviceGuard g(st->ctx->device);
    if (!g.ok) return BH_ENODEV;
    int rc = ensure_moe_graph(st);
    if (rc != BH_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t bytes = (size_t)st->cfg.n_tok * st->cfg.n_embd * sizeof(float);
    if (cudaMemcpyAsync(st->h, h, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess) return BH_EIO;
    if (cudaGraphLaunch(st->exec, s) != cudaSuccess) return BH_EIO;
    return cudaMemcpyAsync(h_out, st->h, bytes, cudaMemcpyDeviceToDevice, s) == cudaSuccess ? BH_OK : BH_EIO;
}

int bh_moe_stack_step_host(bh_moe_stack* st, const float* host_h, float* host_h_out) {
    if (!st || !host_h || !host_h_out) return BH_EINVAL;
    DeviceGuard g(st->ctx->device);
    if (!g.ok) return BH_ENODEV;
    int rc = ensure_moe_graph(st);
    if (rc != BH_OK) return rc;
    const size_t bytes = (size_t)st->cfg.n_tok * st->cfg.n_embd * sizeof(float);
    std::memcpy(st->host_h, host_h, bytes);
    if (cudaMemcpyAsync(st->h, st->host_h, bytes, cudaMemcpyHostToDevice, st->stream) != cudaSuccess ||
        cudaGraphLaunch(st->exec, st->stream) != cudaSuccess ||
        cudaMemcpyAsync(st->host_h, st->h, bytes, cudaMemcpyDeviceToHost, st->stream) != cudaSuccess ||
        cudaStreamSynchronize(st->stream) != cudaSuccess)
        return BH_EIO;
    std::memcpy(host_h_out, st->host_h, bytes);
    return BH_OK;
}

int bh_moe_stack_info(bh_moe_stack* st, int64_t* weight_bytes, int64_t* step_bytes, int64_t* launches) {
    if (!st) return BH_EINVAL;
    DeviceGuard g(st->ctx->device);
    if (!g.ok) return BH_ENODEV;
    const bh_moe_config& c = st->cfg;
    if (weight_bytes) *weight_bytes = (int64_t)c.n_layer * (int64_t)(2 * st->gate_bytes + st->down_bytes);
    if (launches) *launches = (int64_t)c.n_layer;
    if (step_bytes) {
        const size_t n = (size_t)c.n_layer * c.n_tok * c.k;
        std::vector<int32_t> ids(n);
        if (cudaStreamSynchronize(st->stream) != cudaSuccess ||
            cudaMemcpy(ids.data(), st->ids, n * sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
            return BH_EIO;
        const int64_t per_expert = (int64_t)(2 * st->gate_bytes + st->down_bytes) / c.n_expert;
        const int64_t pairs = (int64_t)c.n_tok * c.k;
        // per layer: the distinct experts' weights, h read, gate|up written
        // and read back, expert outputs written and read back, h written
        const int64_t act = (int64_t)c.n_tok * c.n_embd * 4 * 2 + pairs * 2 * c.n_ff * 4 * 2 +
                            pairs * c.n_embd * 4 * 2;
        int64_t total = 0;
        for (int l = 0; l < c.n_layer; ++l) {
            std::vector<char> seen(c.n_expert, 0);
            int u = 0;
            for (int64_t q = 0; q < pairs; ++q) {
                const int e = ids[(size_t)l * pairs + q];
                if (e >= 0 && e < c.n_expert && !seen[e]) { seen[e] = 1; ++u; }
            }
            total += u * per_expert + act;
        }
        *step_bytes = total;
    }
    return BH_OK;
}

int bh_moe_stack_tensor(bh_moe_stack* st, int layer, int which, void** ptr, int64_t* bytes) {
    if (!st || !ptr) return BH_EINVAL;
    const bh_moe_config& c = st->cfg;
    if (which == BH_MOE_HIDDEN) {
        *ptr = st->h;
        if (bytes) *bytes = (int64_t)c.n_tok * c.n_embd * 4;
        return BH_OK;
    }
    if (which == BH_MOE_BARRIER) {
        *ptr = st->gbar;
        if (bytes) *bytes = 256;
        return BH_OK;
    }
    if (layer < 0 || layer >= c.n_layer) return BH_EINVAL;
    switch (which) {
        case BH_MOE_GATE:
        case BH_MOE_UP:
            *ptr = const_cast<uint8_t*>(layer_bank(st, layer, which));
            if (bytes) *bytes = (int64_t)st->gate_bytes;
            return BH_OK;
        case BH_MOE_DOWN:
            *ptr = const_cast<uint8_t*>(layer_bank(st, layer, which));
            if (bytes) *bytes = (int64_t)st->down_bytes;
            return BH_OK;
        case BH_MOE_LOGITS:
            *ptr = st->logits + (size_t)layer * c.n_tok * c.n_expert;
            if (bytes) *bytes = (int64_t)c.n_tok * c.n_expert * 4;
            return BH_OK;
        case BH_MOE_NORM:
            *ptr = st->norm + (size_t)layer * c.n_embd;
            if (bytes) *bytes = (int64_t)c.n_embd * 4;
            return BH_OK;
        case BH_MOE_SELECTED:
            *ptr = st->ids + (size_t)layer * c.n_tok * c.k;
            if (bytes) *bytes = (int64_t)c.n_tok * c.k * 4;
            return BH_OK;
        case BH_MOE_WEIGHTS:
            *ptr = st->wsel + (size_t)layer * c.n_tok * c.k;
            if (bytes) *bytes = (int64_t)c.n_tok * c.k * 4;
            return BH_OK;
        default:
            return BH_EINVAL;
    }
}

}  // extern "C"
