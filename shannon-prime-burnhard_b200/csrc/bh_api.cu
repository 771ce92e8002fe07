// bh_api.cu — the extern "C" boundary (include/bh_q4k.h).
//
// Host-side argument validation happens before any launch; an invalid call
// launches nothing and returns BH_EINVAL. There is no CPU fallback: every
// compute entry point runs the sm_100a kernels or fails.
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

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

// NULL is the CUDA default stream, exactly as in the CUDA runtime; the
// context's own stream serves only the host-buffer entry points.
inline cudaStream_t pick_stream(bh_ctx*, void* stream) { return static_cast<cudaStream_t>(stream); }

int ensure_scratch(bh_ctx* ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return BH_OK;
    if (ctx->scratch) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    const size_t want = (bytes + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
    if (cudaMalloc(&ctx->scratch, want) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    ctx->scratch_bytes = want;
    return BH_OK;
}

int check_matvec_args(bh_ctx* ctx, const void* W, int64_t N, int64_t K, const void* x, int B, const float* y,
                      int fold) {
    if (!ctx) return BH_EINVAL;
    if (N < 0 || K < 0 || K % bh::QK != 0 || B < 0 || B > BH_MAX_BATCH) return BH_EINVAL;
    if (K > (int64_t)1 << 30 || N > (int64_t)1 << 31) return BH_EINVAL;
    if (fold != BH_FOLD_X86 && fold != BH_FOLD_GENERIC) return BH_EINVAL;
    if (N == 0 || B == 0) return BH_OK;
    if (!y || !aligned(y, 4)) return BH_EINVAL;
    if (K == 0) return BH_OK;
    if (!W || !aligned(W, 16) || !x || !aligned(x, 4)) return BH_EINVAL;
    return BH_OK;
}

}  // namespace

namespace bh {
// Choose the grid, shared-memory budget and threads per row for one matvec
// launch.
//  - Batch 1-2 (16-warp CTAs, whose registers fill an SM): one CTA per SM.
//    Matrices with fewer than 32 eight-row tiles per CTA (everything but the
//    LM-head-sized ones) run ctx->tpr_narrow threads per row: 4 for
//    standalone launches (measured on B200 with back-to-back launches:
//    12288x4096 10.4 against 12.5 us at 8, 4096x4096 6.45 against 6.77 us),
//    8 in the decode stack's plan, where twice the working warps, each with
//    half the arithmetic per block, measured faster inside the step. (16 threads per
//    row, 2-row tiles, is available through BH_TUNE_TPR: for the 4096-row
//    matrices of the decode step it puts 14 of 16 warps to work instead of 7,
//    but measured slower there, 1.76 against 1.68 ms per token.)
//  - Larger batches: narrow matrices (fewer than 32 eight-row tiles per SM)
//    run 16-warp CTAs at 8 threads per row, one per SM; the others 8-warp
//    CTAs at 4 threads per row, wide ones (at least one 8-row tile per warp
//    with ctas_per_sm CTAs per SM) that many CTAs per SM, each with
//    smem_cap_small bytes.
// A non-zero sm_budget caps the shared memory one launch holds per SM, so the
// next programmatic launch finds room to start its weight copies early.
int plan_for(bh_ctx* ctx, MatvecParams& p, int grid_override, int fold) {
    const int W = dense_warps(p.B);
    const int act_bytes = p.B * p.nb * ACT_BLOCK_BYTES;
    const bool small = act_bytes <= ctx->small_act_bytes;
    int grid, cap, tpr = 4;
    if (grid_override > 0) {
        grid = grid_override;
        cap = 200 * 1024;
    } else if (p.B <= 2) {
        grid = ctx->num_sms;
        cap = 200 * 1024;
        const int64_t tiles8 = ((p.N + MV_ROWS - 1) / MV_ROWS + grid - 1) / grid;
        if (tiles8 < 2 * W) tpr = ctx->tpr_narrow;
    } else if (ctx->tpr_force == 8 ||
               (ctx->tpr_force == 0 &&
                ((p.N + MV_ROWS - 1) / MV_ROWS + ctx->num_sms - 1) / ctx->num_sms < 2 * DENSE_MAX_WARPS)) {
        // narrow matrices at batch 3-8: 16-warp CTAs, one per SM, 8 threads
        // per row (measured on B200, back-to-back launches at batch 8:
        // 4096x12288 42.5 against 53.2 us, 4096x4096 16.8 against 20.7 us
        // with 8-warp CTAs at 4 threads per row)
        grid = ctx->num_sms;
        cap = 200 * 1024;
        tpr = 8;
    } else {
        const int64_t cps_grid = (int64_t)ctx->num_sms * ctx->ctas_per_sm;
        const int64_t tiles_wide = ((p.N + cps_grid - 1) / cps_grid + MV_ROWS - 1) / MV_ROWS;
        if (small && tiles_wide >= W) {
            grid = (int)cps_grid;
            cap = ctx->smem_cap_small;
        } else {
            grid = ctx->num_sms;
            cap = 200 * 1024;
        }
    }
    if (ctx->sm_budget > 0 && grid_override <= 0) {
        const int per_sm = grid > ctx->num_sms ? (grid + ctx->num_sms - 1) / ctx->num_sms : 1;
        if (per_sm > 1 && per_sm * cap > ctx->sm_budget) grid = ctx->num_sms;
        const int per = grid > ctx->num_sms ? per_sm : 1;
        if (cap * per > ctx->sm_budget) cap = ctx->sm_budget / per;
    }
    if (ctx->tpr_force && p.B <= 2) {
        tpr = 4;
        if (ctx->tpr_force == 8) tpr = 8;
        if (ctx->tpr_force == 16) tpr = (fold == BH_FOLD_X86 && !p.partials) ? 16 : 8;
    }
    const int64_t ntile = (p.N + 32 / tpr - 1) / (32 / tpr);  // CTAs own whole tiles
    if ((int64_t)grid > ntile) grid = (int)ntile;
    const int rc = matvec_plan(p, grid, cap, ctx->stage_bytes, tpr);
    p.prefill = ctx->prefill_stages;
    return rc == BH_OK ? grid : rc;
}

MatvecParams base_params(bh_ctx* ctx, const void* W, int64_t N, int64_t K, int B, float* y) {
    MatvecParams p;
    std::memset(&p, 0, sizeof(p));
    p.w[0] = p.w[1] = p.w[2] = static_cast<const uint8_t*>(W);
    p.seg_end[0] = p.seg_end[1] = p.seg_end[2] = N;
    p.N = N;
    p.K = (int)K;
    p.nb = (int)(K / bh::QK);
    p.B = B;
    p.y = y;
    p.ldy = N;
    p.status = ctx->d_status;
#ifdef BH_TRACE
    p.trace = ctx->trace;
#endif
    return p;
}

void register_barrier_words(bh_ctx* ctx, void* words) {
    std::lock_guard<std::mutex> lock(ctx->barrier_mu.m);
    ctx->barrier_words.push_back(words);
}

void unregister_barrier_words(bh_ctx* ctx, void* words) {
    std::lock_guard<std::mutex> lock(ctx->barrier_mu.m);
    for (size_t i = 0; i < ctx->barrier_words.size(); ++i)
        if (ctx->barrier_words[i] == words) {
            ctx->barrier_words.erase(ctx->barrier_words.begin() + (long)i);
            return;
        }
}

int run_matvec(bh_ctx* ctx, MatvecParams& p, int fold, int src, int epi, cudaStream_t s, bool pdl) {
    const int grid = plan_for(ctx, p, 0, fold);
    if (grid < 0) return grid;
    LaunchOpts o;
    o.stream = s;
    o.grid = grid;
    o.pdl = pdl;
    return launch_matvec(p, fold, src, epi, o);
}
}  // namespace bh

namespace {
using bh::base_params;
using bh::plan_for;
using bh::ACT_BLOCK_BYTES;
using bh::MV_ROWS;
inline int run_matvec(bh_ctx* ctx, bh::MatvecParams& p, int fold, int src, int epi, cudaStream_t s) {
    return bh::run_matvec(ctx, p, fold, src, epi, s, ctx->api_pdl);
}
}  // namespace

extern "C" {

int bh_version(void) { return (1 << 16) | 0; }

const char* bh_strerror(int code) {
    switch (code) {
        case BH_OK: return "ok";
        case BH_EIO: return "CUDA launch or runtime failure";
        case BH_ENOMEM: return "device allocation failed";
        case BH_ENODEV: return "no such CUDA device";
        case BH_EINVAL: return "invalid argument";
        case BH_ETIMEDOUT: return "a bounded device-side wait timed out";
        default: return "unknown status";
    }
}

int bh_init(int device, bh_ctx** out) {
    if (!out) return BH_EINVAL;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return BH_ENODEV;
    }
    DeviceGuard g(device);
    if (!g.ok) return BH_ENODEV;
    bh_ctx* c = new bh_ctx();
    c->device = device;
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    const size_t ncand = (size_t)c->num_sms * 4 * BH_MAX_BATCH;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->d_status, sizeof(int)) != cudaSuccess ||
        cudaMemset(c->d_status, 0, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->cand_val, ncand * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&c->cand_idx, ncand * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        if (c->stream) cudaStreamDestroy(c->stream);
        if (c->d_status) cudaFree(c->d_status);
        if (c->cand_val) cudaFree(c->cand_val);
        if (c->cand_idx) cudaFree(c->cand_idx);
        delete c;
        return BH_ENOMEM;
    }
    *out = c;
    return BH_OK;
}

int bh_free(bh_ctx* ctx) {
    if (!ctx) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->moe_scratch) cudaFree(ctx->moe_scratch);
    cudaFree(ctx->cand_val);
    cudaFree(ctx->cand_idx);
    cudaFree(ctx->d_status);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return BH_OK;
}

#ifdef BH_TRACE
// Timeline probe target (trace builds only; not part of the public header).
int bh_trace_buffer(bh_ctx* ctx, void* dev_buf) {
    if (!ctx) return BH_EINVAL;
    ctx->trace = static_cast<int64_t*>(dev_buf);
    return BH_OK;
}
#endif

int bh_tune(bh_ctx* ctx, int key, int value) {
    if (!ctx) return BH_EINVAL;
    switch (key) {
        case BH_TUNE_CTAS_PER_SM:
            if (value < 1 || value > 4) return BH_EINVAL;
            ctx->ctas_per_sm = value;
            return BH_OK;
        case BH_TUNE_STAGE_BYTES:
            if (value < bh::Q4K_BYTES || value > 65536) return BH_EINVAL;
            ctx->stage_bytes = value;
            ctx->moe_stage_bytes = value;
            return BH_OK;
        case BH_TUNE_TPR:
            if (value != 0 && value != 4 && value != 8 && value != 16) return BH_EINVAL;
            ctx->tpr_force = value;
            return BH_OK;
        case BH_TUNE_SMEM_CAP:
            if (value < 32 * 1024 || value > 200 * 1024) return BH_EINVAL;
            ctx->smem_cap_small = value;
            return BH_OK;
        case BH_TUNE_PDL:
            if (value != 0 && value != 1) return BH_EINVAL;
            ctx->api_pdl = value != 0;
            return BH_OK;
        case BH_TUNE_PREFILL:
            if (value < -1 || value > 8) return BH_EINVAL;
            ctx->prefill_stages = value;
            return BH_OK;
        case BH_TUNE_SMALL_ACT:
            if (value < 0 || value > 128 * 1024) return BH_EINVAL;
            ctx->small_act_bytes = value;
            return BH_OK;
        case BH_TUNE_SM_BUDGET:
            if (value != 0 && (value < 48 * 1024 || value > 228 * 1024)) return BH_EINVAL;
            ctx->sm_budget = value;
            return BH_OK;
        case BH_TUNE_PREFETCH_MB:
            if (value < -1 || value > 120) return BH_EINVAL;
            ctx->prefetch_bytes = value < 0 ? -1 : (int64_t)value << 20;
            return BH_OK;
        case BH_TUNE_BARRIER_WAIT:
            if (value < 16 || value > 31) return BH_EINVAL;
            ctx->barrier_wait_cycles = 1ll << value;
            return BH_OK;
        default:
            return BH_EINVAL;
    }
}

int bh_ctx_device(bh_ctx* ctx) { return ctx ? ctx->device : BH_EINVAL; }

int bh_device_status(bh_ctx* ctx, int clear) {
    if (!ctx) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    if (cudaDeviceSynchronize() != cudaSuccess) return BH_EIO;
    int st = 0;
    if (cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return BH_EIO;
    if (clear && st) cudaMemset(ctx->d_status, 0, sizeof(int));
    if (clear && st == bh::ST_TIMEOUT) {
        // CTAs that gave up on a grid barrier left their arrivals counted:
        // start every barrier of this context from zero again
        std::lock_guard<std::mutex> lock(ctx->barrier_mu.m);
        for (void* w : ctx->barrier_words)
            if (cudaMemset(w, 0, 256) != cudaSuccess) return BH_EIO;
        if (cudaDeviceSynchronize() != cudaSuccess) return BH_EIO;
    }
    if (st == bh::ST_TIMEOUT) return BH_ETIMEDOUT;
    if (st != 0) return BH_EINVAL;
    return BH_OK;
}

int bh_q8k_quantize(bh_ctx* ctx, const float* x, int64_t K, int B, void* x_q8k, void* stream) {
    if (!ctx || K < 0 || K % bh::QK != 0 || B < 0) return BH_EINVAL;
    if (K == 0 || B == 0) return BH_OK;
    if (!x || !aligned(x, 16) || !x_q8k || !aligned(x_q8k, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    return bh::launch_q8k_quantize(x, K, B, static_cast<uint8_t*>(x_q8k), ctx->d_status,
                                   pick_stream(ctx, stream));
}

int bh_q4k_matvec(bh_ctx* ctx, const void* W_q4k, int64_t N, int64_t K, const void* x_q8k, int B, float* y,
                  int32_t* partials_opt, int fold, void* stream) {
    int rc = check_matvec_args(ctx, W_q4k, N, K, x_q8k, B, y, fold);
    if (rc != BH_OK || N == 0 || B == 0) return rc;
    if (partials_opt && !aligned(partials_opt, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    if (K == 0) return cudaMemsetAsync(y, 0, sizeof(float) * (size_t)N * B, s) == cudaSuccess ? BH_OK : BH_EIO;
    bh::MatvecParams p = base_params(ctx, W_q4k, N, K, B, y);
    p.xq = static_cast<const uint8_t*>(x_q8k);
    p.partials = partials_opt;
    return run_matvec(ctx, p, fold, bh::ACT_Q8K, bh::EPI_STORE, s);
}

int bh_q4k_matvec_f32(bh_ctx* ctx, const void* W_q4k, int64_t N, int64_t K, const float* x, int B, float* y,
                      int fold, void* stream) {
    int rc = check_matvec_args(ctx, W_q4k, N, K, x, B, y, fold);
    if (rc != BH_OK || N == 0 || B == 0) return rc;
    if (K > 0 && !aligned(x, 16)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    if (K == 0) return cudaMemsetAsync(y, 0, sizeof(float) * (size_t)N * B, s) == cudaSuccess ? BH_OK : BH_EIO;
    bh::MatvecParams p = base_params(ctx, W_q4k, N, K, B, y);
    p.xf = x;
    return run_matvec(ctx, p, fold, bh::ACT_F32, bh::EPI_STORE, s);
}

int bh_q4k_quantize(bh_ctx* ctx, const float* w, int64_t N, int64_t K, void* W_q4k, void* stream) {
    if (!ctx || N < 0 || K < 0 || K % bh::QK != 0) return BH_EINVAL;
    if (N == 0 || K == 0) return BH_OK;
    if (!w || !aligned(w, 16) || !W_q4k || !aligned(W_q4k, 4)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    return bh::launch_q4k_quantize(w, N, K, static_cast<uint8_t*>(W_q4k), pick_stream(ctx, stream));
}

int bh_q4k_dequantize(bh_ctx* ctx, const void* W_q4k, int64_t N, int64_t K, float* w, void* stream) {
    if (!ctx || N < 0 || K < 0 || K % bh::QK != 0) return BH_EINVAL;
    if (N == 0 || K == 0) return BH_OK;
    if (!w || !aligned(w, 16) || !W_q4k || !aligned(W_q4k, 2)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    return bh::launch_q4k_dequantize(static_cast<const uint8_t*>(W_q4k), N, K, w, pick_stream(ctx, stream));
}

int bh_q4k_lmhead_argmax(bh_ctx* ctx, const void* W_q4k, int64_t N, int64_t K, const float* x, int B,
                         float* logits_opt, int32_t* tok_out, float* max_opt, int fold, void* stream) {
    if (!ctx || !tok_out || !aligned(tok_out, 4) || N < 1 || K < bh::QK || B < 1) return BH_EINVAL;
    if (N > INT32_MAX) return BH_EINVAL;
    int rc = check_matvec_args(ctx, W_q4k, N, K, x, B, logits_opt ? logits_opt : (const float*)tok_out, fold);
    if (rc != BH_OK) return rc;
    if (!aligned(x, 16) || (max_opt && !aligned(max_opt, 4))) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    bh::MatvecParams p = base_params(ctx, W_q4k, N, K, B, logits_opt);
    p.xf = x;
    p.cand_val = ctx->cand_val;
    p.cand_idx = ctx->cand_idx;
    const int grid = plan_for(ctx, p, 0, fold);
    if (grid < 0) return grid;
    bh::LaunchOpts o;
    o.stream = s;
    o.grid = grid;
    o.pdl = ctx->api_pdl;
    if ((rc = bh::launch_matvec(p, fold, bh::ACT_F32, bh::EPI_ARGMAX, o)) != BH_OK) return rc;
    return bh::launch_argmax_finish(ctx->cand_val, ctx->cand_idx, grid, B, tok_out, max_opt, s, false);
}

int bh_q4k_mul_mat_host(bh_ctx* ctx, const void* W_q4k, int64_t N, int64_t K, const float* host_x, int B,
                        float* host_y, int fold) {
    int rc = check_matvec_args(ctx, W_q4k, N, K, host_x, B, host_y, fold);
    if (rc != BH_OK || N == 0 || B == 0) return rc;
    DeviceGuard g(ctx->device);
    const size_t xb = sizeof(float) * (size_t)B * K, yb = sizeof(float) * (size_t)B * N;
    const size_t xoff = 0, yoff = (xb + 255) & ~(size_t)255;
    if ((rc = ensure_scratch(ctx, yoff + yb)) != BH_OK) return rc;
    float* dx = reinterpret_cast<float*>(ctx->scratch + xoff);
    float* dy = reinterpret_cast<float*>(ctx->scratch + yoff);
    cudaStream_t s = ctx->stream;
    if (K > 0 && cudaMemcpyAsync(dx, host_x, xb, cudaMemcpyHostToDevice, s) != cudaSuccess) return BH_EIO;
    if (K == 0) {
        if (cudaMemsetAsync(dy, 0, yb, s) != cudaSuccess) return BH_EIO;
    } else {
        bh::MatvecParams p = base_params(ctx, W_q4k, N, K, B, dy);
        p.xf = dx;
        if ((rc = run_matvec(ctx, p, fold, bh::ACT_F32, bh::EPI_STORE, s)) != BH_OK) return rc;
    }
    if (cudaMemcpyAsync(host_y, dy, yb, cudaMemcpyDeviceToHost, s) != cudaSuccess) return BH_EIO;
    if (cudaStreamSynchronize(s) != cudaSuccess) return BH_EIO;
    return BH_OK;
}

void bh_ggml_vec_dot_q4_K_q8_K(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy, size_t by,
                               int nrc) {
    (void)bs;
    (void)bx;
    (void)by;
    static std::mutex mu;
    static bh_ctx* gctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!s) return;
    *s = 0.f;
    if (nrc != 1 || n < 0 || n % bh::QK != 0 || !vx || !vy) return;
    if (n == 0) return;
    if (!gctx && bh_init(0, &gctx) != BH_OK) return;
    DeviceGuard g(gctx->device);
    const size_t nb = (size_t)n / bh::QK;
    const size_t wb = nb * bh::Q4K_BYTES, xb = nb * bh::Q8K_BYTES;
    const size_t xo = (wb + 255) & ~(size_t)255, yo = (xo + xb + 255) & ~(size_t)255;
    if (ensure_scratch(gctx, yo + 256) != BH_OK) return;
    cudaStream_t st = gctx->stream;
    cudaMemcpyAsync(gctx->scratch, vx, wb, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(gctx->scratch + xo, vy, xb, cudaMemcpyHostToDevice, st);
    bh::MatvecParams p = base_params(gctx, gctx->scratch, 1, n, 1, reinterpret_cast<float*>(gctx->scratch + yo));
    p.xq = gctx->scratch + xo;
    if (run_matvec(gctx, p, BH_FOLD_X86, bh::ACT_Q8K, bh::EPI_STORE, st) != BH_OK) return;
    cudaMemcpyAsync(s, gctx->scratch + yo, sizeof(float), cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
}

}  // extern "C"
