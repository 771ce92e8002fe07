// decode_stack.cu — a Qwen3-8B-shaped decode step built on the Q4_K matvec:
// the caller of the hot path, restating the reference engine's per-token
// block (desktop/engine/src/forward.cpp:2663-2854 build_block_decode; LM
// head :3413; argmax engine.cpp:36-43) for one sequence at batch 1.
//
// Per layer (5 launches, all with programmatic dependent launch, the whole
// step captured once into a CUDA graph):
//   1. QKV matvec   : x = RMSNorm(h) * attn_norm quantized to Q8_K in the
//                     prologue; rows = [Wq; Wk; Wv] as three segments
//   2. attention    : per query head: q/k RMSNorm (Qwen3), NeoX RoPE, KV
//                     append at `pos`, softmax attention over 0..pos (GQA)
//   3. O matvec     : x = attn (quantized in the prologue), h += Wo x
//   4. gate/up      : x = RMSNorm(h) * ffn_norm, rows = [Wg; Wu]
//   5. down matvec  : x = silu(gate) * up (quantized in the prologue), h += Wd x
// then the LM head (RMSNorm * out_norm, logits, per-CTA argmax candidates)
// and the argmax finisher.
//
// All weights are random-init (seeded N(0, 0.02)) and quantized to Q4_K on
// the device by the bit-exact Q4_K quantizer.
#include <cmath>
#include <cstring>
#include <new>

#include <vector>

#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace bh {

// ---------------------------------------------------------------------------
// seeded normal fill: element e = mean + std * z(seed, e), splitmix64 ->
// two 53-bit uniforms -> Box-Muller in double (the oracle's generator).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
__device__ __forceinline__ double unit53(uint64_t seed, uint64_t ctr) {
    return (double)(mix64(seed + (ctr + 1u) * 0x9e3779b97f4a7c15ULL) >> 11) * 0x1.0p-53;
}

__global__ void fill_normal_kernel(float* out, int64_t n, int64_t first, uint64_t seed, double mean, double stddev) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    const int64_t e = first + t, pair = e >> 1;
    const double u1 = 1.0 - unit53(seed, (uint64_t)(2 * pair));
    const double u2 = unit53(seed, (uint64_t)(2 * pair + 1));
    const double r = sqrt(-2.0 * log(u1));
    const double two_pi = 6.283185307179586476925286766559;
    const double z = (e & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
    out[t] = (float)(mean + stddev * z);
}

int fill_normal(float* out, int64_t n, int64_t first, uint64_t seed, double mean, double stddev, cudaStream_t s) {
    if (n <= 0) return BH_OK;
    fill_normal_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(out, n, first, seed, mean, stddev);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

// ---------------------------------------------------------------------------
// attention for one decode token, one CTA per query head, head_dim threads
// ---------------------------------------------------------------------------
struct AttnParams {
    const float* qkv;        // [q_dim | kv_dim | kv_dim]
    float* kc;               // K cache [n_ctx][n_head_kv][head_dim]
    float* vc;               // V cache
    const float* q_norm;     // [head_dim]
    const float* k_norm;     // [head_dim]
    const int* pos;          // device scalar: position of this token (set before the step)
    const float* rope_inv_freq;  // [head_dim / 2]: theta^(-2j / head_dim)
    float* out;              // [q_dim]
    int n_head, n_head_kv, head_dim, n_ctx;
    float eps, theta;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
    // fixed-order reduction: warp butterflies, then warps in order
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t = __fadd_rn(t, red[i]);
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
    for (int i = 1; i < nw; ++i) t = fmaxf(t, red[i]);
    return t;
}

// One CTA of ATTN_THREADS per query head (head_dim 128: lane l of a warp
// holds dims 4l..4l+3 of a row). Positions are dealt round-robin to the
// warps, ATTN_U per warp per round; each warp reads whole K / V rows with one
// coalesced 512-byte load. The K / V history (positions before this token)
// does not depend on the previous kernel, so the first round's rows are
// loaded before the programmatic-launch wait and arrive while the QKV
// projection finishes. Per-warp partial outputs are combined in warp order.
constexpr int ATTN_THREADS = 256;
constexpr int ATTN_WARPS = ATTN_THREADS / 32;
constexpr int ATTN_HD = 128;
#ifndef BH_ATTN_U
#define BH_ATTN_U 16
#endif
constexpr int ATTN_U = BH_ATTN_U;  // positions per warp per round (16: 128 positions per round)

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const AttnParams a) {
    extern __shared__ float s_scores[];  // [n_ctx]
    __shared__ float sq[ATTN_HD], sk[ATTN_HD], sv[ATTN_HD], red[ATTN_WARPS];
    __shared__ float4 s_part[ATTN_WARPS][ATTN_HD / 4];
    constexpr int U = ATTN_U;
    const int h = blockIdx.x, tid = threadIdx.x, HD = ATTN_HD, half = HD / 2;
    const int group = a.n_head / a.n_head_kv, g = h / group;
    const int q_dim = a.n_head * HD, kv_dim = a.n_head_kv * HD;
    const int pos = *a.pos;
    const int lane = tid & 31, w = tid >> 5;
    const int64_t row_stride = (int64_t)a.n_head_kv * HD;
    const float* kbase = a.kc + (int64_t)g * HD;
    const float* vbase = a.vc + (int64_t)g * HD;

    // before the wait: the first round of K / V history rows and the weights
    float4 kpre[U], vpre[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int t = w + u * ATTN_WARPS;
        kpre[u] = t < pos ? reinterpret_cast<const float4*>(kbase + (int64_t)t * row_stride)[lane] : f4_zero();
        vpre[u] = t < pos ? reinterpret_cast<const float4*>(vbase + (int64_t)t * row_stride)[lane] : f4_zero();
    }
    float qn = 0.f, kn = 0.f, inv_freq = 0.f;
    if (tid < HD) {
        qn = a.q_norm[tid];
        kn = a.k_norm[tid];
        inv_freq = a.rope_inv_freq[tid < half ? tid : tid - half];
    }
    pdl_trigger();
    pdl_wait();

    // this head's q, k, v (threads 0..HD-1), per-head RMSNorm, NeoX RoPE
    float q = 0.f, k = 0.f, v = 0.f;
    if (tid < HD) {
        q = a.qkv[h * HD + tid];
        k = a.qkv[q_dim + g * HD + tid];
        v = a.qkv[q_dim + kv_dim + g * HD + tid];
    }
    const float sq_q = block_sum(__fmul_rn(q, q), red);
    const float sq_k = block_sum(__fmul_rn(k, k), red);
    const float rq = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq_q, (float)HD), a.eps)));
    const float rk = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq_k, (float)HD), a.eps)));
    if (tid < HD) {
        q = __fmul_rn(__fmul_rn(q, rq), qn);
        k = __fmul_rn(__fmul_rn(k, rk), kn);
        sq[tid] = q;
        sk[tid] = k;
        sv[tid] = v;
    }
    __syncthreads();
    float qr = 0.f, kr = 0.f;
    if (tid < HD) {
        const float ang = (float)pos * inv_freq;
        float sn, cs;
        sincosf(ang, &sn, &cs);
        if (tid < half) {
            qr = __fsub_rn(__fmul_rn(q, cs), __fmul_rn(sq[tid + half], sn));
            kr = __fsub_rn(__fmul_rn(k, cs), __fmul_rn(sk[tid + half], sn));
        } else {
            qr = __fadd_rn(__fmul_rn(q, cs), __fmul_rn(sq[tid - half], sn));
            kr = __fadd_rn(__fmul_rn(k, cs), __fmul_rn(sk[tid - half], sn));
        }
    }
    __syncthreads();
    if (tid < HD) {
        sq[tid] = qr;
        sk[tid] = kr;
        if (h % group == 0) {
            a.kc[(int64_t)pos * row_stride + g * HD + tid] = kr;
            a.vc[(int64_t)pos * row_stride + g * HD + tid] = v;
        }
    }
    __syncthreads();
    // scores: warp w takes positions w, w + ATTN_WARPS, ...; this token's own
    // K comes from shared memory
    const float4 q4 = reinterpret_cast<const float4*>(sq)[lane];
    const float scale = __fdiv_rn(1.f, __fsqrt_rn((float)HD));
    for (int t0 = w; t0 <= pos; t0 += ATTN_WARPS * U) {
        const bool first = t0 == w;
        float4 kv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = t0 + u * ATTN_WARPS;
            kv[u] = t > pos    ? f4_zero()
                    : t == pos ? reinterpret_cast<const float4*>(sk)[lane]
                    : first    ? kpre[u]
                               : reinterpret_cast<const float4*>(kbase + (int64_t)t * row_stride)[lane];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = t0 + u * ATTN_WARPS;
            float dot = __fadd_rn(__fadd_rn(__fmul_rn(q4.x, kv[u].x), __fmul_rn(q4.y, kv[u].y)),
                                  __fadd_rn(__fmul_rn(q4.z, kv[u].z), __fmul_rn(q4.w, kv[u].w)));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, off));
            if (lane == 0 && t <= pos) s_scores[t] = __fmul_rn(dot, scale);
        }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int t = tid; t <= pos; t += ATTN_THREADS) mx = fmaxf(mx, s_scores[t]);
    mx = block_max(mx, red);
    float se = 0.f;
    for (int t = tid; t <= pos; t += ATTN_THREADS) {
        const float e = expf(__fsub_rn(s_scores[t], mx));
        s_scores[t] = e;
        se = __fadd_rn(se, e);
    }
    se = block_sum(se, red);  // (its barrier publishes s_scores)
    // weighted V: warp w accumulates its positions for dims 4*lane..4*lane+3
    float4 o = f4_zero();
    for (int t0 = w; t0 <= pos; t0 += ATTN_WARPS * U) {
        const bool first = t0 == w;
        float4 vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = t0 + u * ATTN_WARPS;
            vv[u] = t > pos    ? f4_zero()
                    : t == pos ? reinterpret_cast<const float4*>(sv)[lane]
                    : first    ? vpre[u]
                               : reinterpret_cast<const float4*>(vbase + (int64_t)t * row_stride)[lane];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = t0 + u * ATTN_WARPS;
            const float p = t <= pos ? s_scores[t] : 0.f;
            o.x = __fadd_rn(o.x, __fmul_rn(p, vv[u].x));
            o.y = __fadd_rn(o.y, __fmul_rn(p, vv[u].y));
            o.z = __fadd_rn(o.z, __fmul_rn(p, vv[u].z));
            o.w = __fadd_rn(o.w, __fmul_rn(p, vv[u].w));
        }
    }
    s_part[w][lane] = o;
    __syncthreads();
    if (tid < HD / 4) {
        float4 r = s_part[0][tid];
        for (int i = 1; i < ATTN_WARPS; ++i) {
            const float4 pi = s_part[i][tid];
            r.x = __fadd_rn(r.x, pi.x);
            r.y = __fadd_rn(r.y, pi.y);
            r.z = __fadd_rn(r.z, pi.z);
            r.w = __fadd_rn(r.w, pi.w);
        }
        float4 res = make_float4(__fdiv_rn(r.x, se), __fdiv_rn(r.y, se), __fdiv_rn(r.z, se), __fdiv_rn(r.w, se));
        reinterpret_cast<float4*>(a.out + h * HD)[tid] = res;
    }
}

}  // namespace bh

// ---------------------------------------------------------------------------
// the stack object
// ---------------------------------------------------------------------------
struct bh_stack {
    bh_ctx* ctx = nullptr;
    // launch plan of the step's layer matvecs: a copy of ctx whose tuning
    // leaves room on every SM for the next launch (see bh_stack_create)
    bh_ctx plan;
    bh_stack_config cfg;
    cudaStream_t stream = nullptr;
    // one allocation for all Q4_K weights
    uint8_t* wbuf = nullptr;
    size_t wbytes = 0;
    const uint8_t** wq = nullptr;   // [n_layer * BH_W_PER_LAYER] then the LM head
    float* fbuf = nullptr;          // norms, KV caches, activations
    float *attn_norm, *ffn_norm, *q_norm, *k_norm, *out_norm;
    float* rope_inv_freq;           // [head_dim / 2]
    float *kc, *vc;
    float *x_in, *h, *qkv, *attn, *gu, *logits, *cand_val;
    int32_t *cand_idx, *tok;
    int* pos;
    int32_t* host_tok = nullptr;    // pinned
    float* host_x = nullptr;        // pinned staging for the host-buffer call
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int lm_grid = 0;
    int64_t step_bytes = 0;         // algorithmic bytes of one decode step
    int64_t launches = 0;           // kernel launches in one step
};

namespace {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int check_cfg(const bh_stack_config* c) {
    if (!c) return BH_EINVAL;
    if (c->n_layer < 1 || c->n_embd < 256 || c->n_embd % 256 || c->n_ff < 256 || c->n_ff % 256) return BH_EINVAL;
    if (c->head_dim != bh::ATTN_HD) return BH_EINVAL;  // the attention kernel is written for 128
    if (c->n_head < 1 || c->n_head_kv < 1 || c->n_head % c->n_head_kv) return BH_EINVAL;
    if ((c->n_head * c->head_dim) % 256 || c->n_vocab < 1 || c->n_ctx < 1 || c->n_ctx > 8192) return BH_EINVAL;
    return BH_OK;
}

void mat_dims(const bh_stack_config& c, int which, int64_t* rows, int64_t* cols) {
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    switch (which) {
        case BH_W_Q: *rows = qd; *cols = c.n_embd; break;
        case BH_W_K: *rows = kvd; *cols = c.n_embd; break;
        case BH_W_V: *rows = kvd; *cols = c.n_embd; break;
        case BH_W_O: *rows = c.n_embd; *cols = qd; break;
        case BH_W_GATE: *rows = c.n_ff; *cols = c.n_embd; break;
        case BH_W_UP: *rows = c.n_ff; *cols = c.n_embd; break;
        case BH_W_DOWN: *rows = c.n_embd; *cols = c.n_ff; break;
        default: *rows = c.n_vocab; *cols = c.n_embd; break;  // LM head
    }
}

uint64_t tensor_seed(uint64_t seed, int layer, int which) {
    uint64_t z = seed ^ (0x51ed2701a3b4c5d6ULL + (uint64_t)layer * 0x9e3779b97f4a7c15ULL + (uint64_t)which * 0xd6e8feb86659fd93ULL);
    z = (z ^ (z >> 31)) * 0x7fb5d329728ea185ULL;
    return z ^ (z >> 27);
}

int stack_matvec(bh_stack* st, bh::MatvecParams& p, int src, int epi, bool pdl) {
    return bh::run_matvec(&st->plan, p, BH_FOLD_X86, src, epi, st->stream, pdl);
}

// Attention of layer l over positions 0..pos (one CTA per query head).
int launch_attn(bh_stack* st, int l, bool pdl) {
    const bh_stack_config& c = st->cfg;
    const int64_t kvd = (int64_t)c.n_head_kv * c.head_dim;
    bh::AttnParams a;
    a.qkv = st->qkv;
    a.kc = st->kc + (size_t)l * c.n_ctx * kvd;
    a.vc = st->vc + (size_t)l * c.n_ctx * kvd;
    a.q_norm = st->q_norm + (size_t)l * c.head_dim;
    a.k_norm = st->k_norm + (size_t)l * c.head_dim;
    a.pos = st->pos;
    a.out = st->attn;
    a.n_head = c.n_head;
    a.n_head_kv = c.n_head_kv;
    a.head_dim = c.head_dim;
    a.n_ctx = c.n_ctx;
    a.eps = c.rms_eps;
    a.theta = c.rope_theta;
    a.rope_inv_freq = st->rope_inv_freq;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)c.n_head);
    cfg.blockDim = dim3((unsigned)bh::ATTN_THREADS);
    cfg.dynamicSmemBytes = sizeof(float) * (size_t)c.n_ctx;
    cfg.stream = st->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    static bool attr_set = false;
    if (!attr_set) {
        // the same shared-memory carveout as the matvecs around it
        if (cudaFuncSetAttribute(bh::attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return BH_EIO;
        attr_set = true;
    }
    return cudaLaunchKernelEx(&cfg, bh::attn_decode_kernel, a) == cudaSuccess ? BH_OK : BH_EIO;
}

// Enqueue one decode step on st->stream (captured into the graph).
int enqueue_step(bh_stack* st) {
    const bh_stack_config& c = st->cfg;
    bh_ctx* ctx = st->ctx;
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    int rc;
    if (cudaMemcpyAsync(st->h, st->x_in, sizeof(float) * c.n_embd, cudaMemcpyDeviceToDevice, st->stream) != cudaSuccess)
        return BH_EIO;
    st->step_bytes = 0;
    st->launches = 0;
    auto account = [&](const bh::MatvecParams& p, int b_in_bytes) {
        st->step_bytes += p.N * (int64_t)p.nb * bh::Q4K_BYTES + b_in_bytes + p.N * 4;
        st->launches += 1;
    };
    for (int l = 0; l < c.n_layer; ++l) {
        const uint8_t* const* W = st->wq + (size_t)l * BH_W_PER_LAYER;
        // 1. QKV
        bh::MatvecParams p = bh::base_params(ctx, W[BH_W_Q], qd + 2 * kvd, c.n_embd, 1, st->qkv);
        p.w[1] = W[BH_W_K];
        p.w[2] = W[BH_W_V];
        p.seg_end[0] = qd;
        p.seg_end[1] = qd + kvd;
        p.seg_end[2] = qd + 2 * kvd;
        p.xf = st->h;
        p.gamma = st->attn_norm + (size_t)l * c.n_embd;
        p.eps = c.rms_eps;
        if ((rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, l > 0)) != BH_OK) return rc;
        account(p, c.n_embd * 4);
        // 2. attention
        if ((rc = launch_attn(st, l, true)) != BH_OK) return rc;
        st->launches += 1;
        // 3. O projection, residual add
        p = bh::base_params(ctx, W[BH_W_O], c.n_embd, qd, 1, st->h);
        p.xf = st->attn;
        if ((rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, true)) != BH_OK) return rc;
        account(p, (int)qd * 4);
        // 4. gate / up
        p = bh::base_params(ctx, W[BH_W_GATE], 2 * (int64_t)c.n_ff, c.n_embd, 1, st->gu);
        p.w[1] = p.w[2] = W[BH_W_UP];
        p.seg_end[0] = c.n_ff;
        p.seg_end[1] = p.seg_end[2] = 2 * (int64_t)c.n_ff;
        p.xf = st->h;
        p.gamma = st->ffn_norm + (size_t)l * c.n_embd;
        p.eps = c.rms_eps;
        if ((rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, true)) != BH_OK) return rc;
        account(p, c.n_embd * 4);
        // 5. down, SwiGLU in the prologue, residual add
        p = bh::base_params(ctx, W[BH_W_DOWN], c.n_embd, c.n_ff, 1, st->h);
        p.xf = st->gu;
        if ((rc = stack_matvec(st, p, bh::ACT_F32_SWIGLU, bh::EPI_ADD, true)) != BH_OK) return rc;
        account(p, 2 * c.n_ff * 4);
    }
    // LM head + argmax
    bh::MatvecParams p = bh::base_params(ctx, st->wq[(size_t)c.n_layer * BH_W_PER_LAYER], c.n_vocab, c.n_embd, 1,
                                         st->logits);
    p.xf = st->h;
    p.gamma = st->out_norm;
    p.eps = c.rms_eps;
    p.cand_val = st->cand_val;
    p.cand_idx = st->cand_idx;
    const int grid = bh::plan_for(ctx, p, 0);
    if (grid < 0) return grid;
    st->lm_grid = grid;
    bh::LaunchOpts o;
    o.stream = st->stream;
    o.grid = grid;
    o.pdl = true;
    if ((rc = bh::launch_matvec(p, BH_FOLD_X86, bh::ACT_F32_RMSNORM, bh::EPI_ARGMAX, o)) != BH_OK) return rc;
    account(p, c.n_embd * 4);
    if ((rc = bh::launch_argmax_finish(st->cand_val, st->cand_idx, grid, 1, st->tok, nullptr, st->stream, true)) !=
        BH_OK)
        return rc;
    st->launches += 1;
    return BH_OK;
}

// Launch one op of the step for every layer (or the LM head once), eagerly,
// with the same parameters the step uses.
int enqueue_op(bh_stack* st, int op) {
    const bh_stack_config& c = st->cfg;
    bh_ctx* ctx = st->ctx;
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    int rc = BH_OK;
    if (op == BH_OP_LMHEAD) {
        bh::MatvecParams p = bh::base_params(ctx, st->wq[(size_t)c.n_layer * BH_W_PER_LAYER], c.n_vocab, c.n_embd, 1,
                                             st->logits);
        p.xf = st->h;
        p.gamma = st->out_norm;
        p.eps = c.rms_eps;
        p.cand_val = st->cand_val;
        p.cand_idx = st->cand_idx;
        const int grid = bh::plan_for(ctx, p, 0);
        if (grid < 0) return grid;
        bh::LaunchOpts o;
        o.stream = st->stream;
        o.grid = grid;
        return bh::launch_matvec(p, BH_FOLD_X86, bh::ACT_F32_RMSNORM, bh::EPI_ARGMAX, o);
    }
    if (op == BH_OP_ATTN) {
        for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) rc = launch_attn(st, l, false);
        return rc;
    }
    for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) {
        const uint8_t* const* W = st->wq + (size_t)l * BH_W_PER_LAYER;
        bh::MatvecParams p;
        switch (op) {
            case BH_OP_QKV:
                p = bh::base_params(ctx, W[BH_W_Q], qd + 2 * kvd, c.n_embd, 1, st->qkv);
                p.w[1] = W[BH_W_K];
                p.w[2] = W[BH_W_V];
                p.seg_end[0] = qd;
                p.seg_end[1] = qd + kvd;
                p.seg_end[2] = qd + 2 * kvd;
                p.xf = st->h;
                p.gamma = st->attn_norm + (size_t)l * c.n_embd;
                p.eps = c.rms_eps;
                rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, false);
                break;
            case BH_OP_O:
                p = bh::base_params(ctx, W[BH_W_O], c.n_embd, qd, 1, st->h);
                p.xf = st->attn;
                rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, false);
                break;
            case BH_OP_GATE_UP:
                p = bh::base_params(ctx, W[BH_W_GATE], 2 * (int64_t)c.n_ff, c.n_embd, 1, st->gu);
                p.w[1] = p.w[2] = W[BH_W_UP];
                p.seg_end[0] = c.n_ff;
                p.seg_end[1] = p.seg_end[2] = 2 * (int64_t)c.n_ff;
                p.xf = st->h;
                p.gamma = st->ffn_norm + (size_t)l * c.n_embd;
                p.eps = c.rms_eps;
                rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, false);
                break;
            case BH_OP_DOWN:
                p = bh::base_params(ctx, W[BH_W_DOWN], c.n_embd, c.n_ff, 1, st->h);
                p.xf = st->gu;
                rc = stack_matvec(st, p, bh::ACT_F32_SWIGLU, bh::EPI_ADD, false);
                break;
            default:
                return BH_EINVAL;
        }
    }
    return rc;
}

int ensure_graph(bh_stack* st) {
    if (st->exec) return BH_OK;
    if (cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return BH_EIO;
    const int rc = enqueue_step(st);
    cudaGraph_t g = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(st->stream, &g);
    if (rc != BH_OK || ec != cudaSuccess) {
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

void bh_stack_default_config(bh_stack_config* c) {
    if (!c) return;
    c->n_layer = 36;
    c->n_embd = 4096;
    c->n_head = 32;
    c->n_head_kv = 8;
    c->head_dim = 128;
    c->n_ff = 12288;
    c->n_vocab = 151936;
    c->n_ctx = 128;
    c->rms_eps = 1e-6f;
    c->rope_theta = 1000000.f;
}

int bh_stack_create(bh_ctx* ctx, const bh_stack_config* cfg, uint64_t seed, bh_stack** out) {
    if (!ctx || !out) return BH_EINVAL;
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc != BH_OK) return rc;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return BH_ENODEV;
    bh_stack* st = new (std::nothrow) bh_stack();
    if (!st) return BH_ENOMEM;
    st->ctx = ctx;
    // The layer matvecs follow one another through programmatic launches; the
    // next one can start its weight copies only if it finds room on the SMs.
    // Unless the caller tuned a per-SM budget on ctx, the step therefore plans
    // its layer matvecs within 168 KiB of shared memory per SM with 1152-byte
    // row slices per stage (one 16-warp CTA per SM; the planner picks the
    // threads per row). The LM head, which nothing follows, keeps ctx's plan.
    st->plan = *ctx;
    if (ctx->sm_budget == 0) {
        st->plan.sm_budget = 168 * 1024;
        st->plan.stage_bytes = 1152;
    }
    st->cfg = *cfg;
    const bh_stack_config& c = st->cfg;
    const int nmat = c.n_layer * BH_W_PER_LAYER + 1;
    st->wq = new (std::nothrow) const uint8_t*[nmat];
    if (!st->wq || cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking) != cudaSuccess) {
        bh_stack_free(st);
        return BH_ENOMEM;
    }
    // weights: one allocation, each matrix 256-byte aligned
    size_t off[4096];
    if (nmat > 4096) { bh_stack_free(st); return BH_EINVAL; }
    size_t total = 0, max_mat = 0;
    for (int i = 0; i < nmat; ++i) {
        int64_t r, k;
        mat_dims(c, i < c.n_layer * BH_W_PER_LAYER ? i % BH_W_PER_LAYER : -1, &r, &k);
        off[i] = total;
        const size_t b = (size_t)r * (k / bh::QK) * bh::Q4K_BYTES;
        total = align_up(total + b, 256);
        if (b > max_mat) max_mat = b;
    }
    st->wbytes = total;
    if (cudaMalloc(&st->wbuf, total) != cudaSuccess) {
        cudaGetLastError();
        bh_stack_free(st);
        return BH_ENOMEM;
    }
    for (int i = 0; i < nmat; ++i) st->wq[i] = st->wbuf + off[i];
    // fp32 side buffers
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    const int cand_max = ctx->num_sms * 4;
    size_t fl = 0;
    auto take = [&](int64_t n) { const size_t o = fl; fl = align_up(fl + (size_t)n, 64); return o; };
    const size_t o_an = take((int64_t)c.n_layer * c.n_embd), o_fn = take((int64_t)c.n_layer * c.n_embd);
    const size_t o_qn = take((int64_t)c.n_layer * c.head_dim), o_kn = take((int64_t)c.n_layer * c.head_dim);
    const size_t o_on = take(c.n_embd);
    const size_t o_kc = take((int64_t)c.n_layer * c.n_ctx * kvd), o_vc = take((int64_t)c.n_layer * c.n_ctx * kvd);
    const size_t o_x = take(c.n_embd), o_h = take(c.n_embd), o_qkv = take(qd + 2 * kvd), o_at = take(qd);
    const size_t o_gu = take(2 * (int64_t)c.n_ff), o_lg = take(c.n_vocab), o_cv = take(cand_max);
    const size_t o_ci = take(cand_max), o_tk = take(1), o_ps = take(1), o_rf = take(c.head_dim / 2);
    if (cudaMalloc(&st->fbuf, fl * sizeof(float)) != cudaSuccess ||
        cudaMallocHost(&st->host_tok, sizeof(int32_t)) != cudaSuccess ||
        cudaMallocHost(&st->host_x, sizeof(float) * c.n_embd) != cudaSuccess) {
        cudaGetLastError();
        bh_stack_free(st);
        return BH_ENOMEM;
    }
    cudaMemsetAsync(st->fbuf, 0, fl * sizeof(float), st->stream);
    float* F = st->fbuf;
    st->attn_norm = F + o_an; st->ffn_norm = F + o_fn; st->q_norm = F + o_qn; st->k_norm = F + o_kn;
    st->out_norm = F + o_on; st->kc = F + o_kc; st->vc = F + o_vc; st->x_in = F + o_x; st->h = F + o_h;
    st->qkv = F + o_qkv; st->attn = F + o_at; st->gu = F + o_gu; st->logits = F + o_lg; st->cand_val = F + o_cv;
    st->cand_idx = reinterpret_cast<int32_t*>(F + o_ci);
    st->tok = reinterpret_cast<int32_t*>(F + o_tk);
    st->pos = reinterpret_cast<int*>(F + o_ps);
    st->rope_inv_freq = F + o_rf;
    {
        // NeoX RoPE frequencies theta^(-2j / head_dim), evaluated in double once per stack
        std::vector<float> rf((size_t)c.head_dim / 2);
        for (int j = 0; j < c.head_dim / 2; ++j)
            rf[(size_t)j] = (float)std::exp(-(2.0 * j / c.head_dim) * std::log((double)c.rope_theta));
        if (cudaMemcpyAsync(st->rope_inv_freq, rf.data(), rf.size() * sizeof(float), cudaMemcpyHostToDevice,
                            st->stream) != cudaSuccess ||
            cudaStreamSynchronize(st->stream) != cudaSuccess) {
            bh_stack_free(st);
            return BH_EIO;
        }
    }
    // norm weights ~ 1 + N(0, 0.02)
    if ((rc = bh::fill_normal(st->attn_norm, (int64_t)c.n_layer * c.n_embd, 0, tensor_seed(seed, -1, 1), 1.0, 0.02, st->stream)) ||
        (rc = bh::fill_normal(st->ffn_norm, (int64_t)c.n_layer * c.n_embd, 0, tensor_seed(seed, -1, 2), 1.0, 0.02, st->stream)) ||
        (rc = bh::fill_normal(st->q_norm, (int64_t)c.n_layer * c.head_dim, 0, tensor_seed(seed, -1, 3), 1.0, 0.02, st->stream)) ||
        (rc = bh::fill_normal(st->k_norm, (int64_t)c.n_layer * c.head_dim, 0, tensor_seed(seed, -1, 4), 1.0, 0.02, st->stream)) ||
        (rc = bh::fill_normal(st->out_norm, c.n_embd, 0, tensor_seed(seed, -1, 5), 1.0, 0.02, st->stream))) {
        bh_stack_free(st);
        return rc;
    }
    // Q4_K weights: seeded N(0, 0.02) in fp32 chunks, quantized on the device
    const size_t chunk_floats = (size_t)64 << 20;  // 256 MiB of fp32 per chunk
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, chunk_floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        bh_stack_free(st);
        return BH_ENOMEM;
    }
    for (int i = 0; i < nmat && rc == BH_OK; ++i) {
        const int layer = i < c.n_layer * BH_W_PER_LAYER ? i / BH_W_PER_LAYER : c.n_layer;
        const int which = i < c.n_layer * BH_W_PER_LAYER ? i % BH_W_PER_LAYER : BH_W_PER_LAYER;
        int64_t r, k;
        mat_dims(c, i < c.n_layer * BH_W_PER_LAYER ? which : -1, &r, &k);
        const int64_t rows_per_chunk = (int64_t)(chunk_floats / (size_t)k);
        const uint64_t ts = tensor_seed(seed, layer, which);
        for (int64_t r0 = 0; r0 < r && rc == BH_OK; r0 += rows_per_chunk) {
            const int64_t nr = r - r0 < rows_per_chunk ? r - r0 : rows_per_chunk;
            rc = bh::fill_normal(tmp, nr * k, r0 * k, ts, 0.0, 0.02, st->stream);
            if (rc == BH_OK)
                rc = bh::launch_q4k_quantize(tmp, nr, k,
                                             const_cast<uint8_t*>(st->wq[i]) + (size_t)r0 * (k / bh::QK) * bh::Q4K_BYTES,
                                             st->stream);
        }
    }
    cudaStreamSynchronize(st->stream);
    cudaFree(tmp);
    if (rc != BH_OK || cudaGetLastError() != cudaSuccess) {
        bh_stack_free(st);
        return rc != BH_OK ? rc : BH_EIO;
    }
    *out = st;
    return BH_OK;
}

int bh_stack_free(bh_stack* st) {
    if (!st) return BH_EINVAL;
    if (st->stream) cudaStreamSynchronize(st->stream);
    if (st->exec) cudaGraphExecDestroy(st->exec);
    if (st->graph) cudaGraphDestroy(st->graph);
    if (st->wbuf) cudaFree(st->wbuf);
    if (st->fbuf) cudaFree(st->fbuf);
    if (st->host_tok) cudaFreeHost(st->host_tok);
    if (st->host_x) cudaFreeHost(st->host_x);
    if (st->stream) cudaStreamDestroy(st->stream);
    delete[] st->wq;
    delete st;
    return BH_OK;
}

int bh_stack_set_pos(bh_stack* st, int pos) {
    if (!st || pos < 0 || pos >= st->cfg.n_ctx) return BH_EINVAL;
    return cudaMemcpyAsync(st->pos, &pos, sizeof(int), cudaMemcpyHostToDevice, st->stream) == cudaSuccess &&
                   cudaStreamSynchronize(st->stream) == cudaSuccess
               ? BH_OK
               : BH_EIO;
}

int bh_stack_fill_kv(bh_stack* st, int n_pos, uint64_t seed) {
    if (!st || n_pos < 0 || n_pos > st->cfg.n_ctx) return BH_EINVAL;
    const bh_stack_config& c = st->cfg;
    const int64_t kvd = (int64_t)c.n_head_kv * c.head_dim;
    int rc = BH_OK;
    for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) {
        rc = bh::fill_normal(st->kc + (size_t)l * c.n_ctx * kvd, n_pos * kvd, 0, tensor_seed(seed, l, 100), 0.0, 1.0, st->stream);
        if (rc == BH_OK)
            rc = bh::fill_normal(st->vc + (size_t)l * c.n_ctx * kvd, n_pos * kvd, 0, tensor_seed(seed, l, 101), 0.0, 1.0, st->stream);
    }
    if (cudaStreamSynchronize(st->stream) != cudaSuccess) return BH_EIO;
    return rc;
}

int bh_stack_decode(bh_stack* st, const float* x, int32_t* tok_out, void* stream) {
    if (!st || !x || !tok_out) return BH_EINVAL;
    int rc = ensure_graph(st);
    if (rc != BH_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t xb = sizeof(float) * st->cfg.n_embd;
    if (cudaMemcpyAsync(st->x_in, x, xb, cudaMemcpyDeviceToDevice, s) != cudaSuccess) return BH_EIO;
    if (cudaGraphLaunch(st->exec, s) != cudaSuccess) return BH_EIO;
    if (cudaMemcpyAsync(tok_out, st->tok, sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess) return BH_EIO;
    return BH_OK;
}

int bh_stack_decode_host(bh_stack* st, const float* host_x, int32_t* host_tok) {
    if (!st || !host_x || !host_tok) return BH_EINVAL;
    int rc = ensure_graph(st);
    if (rc != BH_OK) return rc;
    const size_t xb = sizeof(float) * st->cfg.n_embd;
    if (cudaMemcpyAsync(st->x_in, host_x, xb, cudaMemcpyHostToDevice, st->stream) != cudaSuccess) return BH_EIO;
    if (cudaGraphLaunch(st->exec, st->stream) != cudaSuccess) return BH_EIO;
    if (cudaMemcpyAsync(st->host_tok, st->tok, sizeof(int32_t), cudaMemcpyDeviceToHost, st->stream) != cudaSuccess)
        return BH_EIO;
    if (cudaStreamSynchronize(st->stream) != cudaSuccess) return BH_EIO;
    *host_tok = *st->host_tok;
    return BH_OK;
}

int bh_stack_info(bh_stack* st, int64_t* weight_bytes, int64_t* step_bytes, int64_t* launches) {
    if (!st) return BH_EINVAL;
    int rc = ensure_graph(st);
    if (rc != BH_OK) return rc;
    if (weight_bytes) *weight_bytes = (int64_t)st->wbytes;
    if (step_bytes) *step_bytes = st->step_bytes;
    if (launches) *launches = st->launches;
    return BH_OK;
}

int bh_stack_time_op(bh_stack* st, int op, int reps, float* avg_ms, int64_t* bytes_per_launch) {
    if (!st || !avg_ms || reps < 1 || op < BH_OP_QKV || op > BH_OP_ATTN) return BH_EINVAL;
    const bh_stack_config& c = st->cfg;
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    int64_t rows = 0, k = 0, xin = 0;
    switch (op) {
        case BH_OP_QKV: rows = qd + 2 * kvd; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
        case BH_OP_O: rows = c.n_embd; k = qd; xin = qd * 4 + (int64_t)c.n_embd * 4; break;
        case BH_OP_GATE_UP: rows = 2 * (int64_t)c.n_ff; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
        case BH_OP_DOWN: rows = c.n_embd; k = c.n_ff; xin = 2 * (int64_t)c.n_ff * 4 + (int64_t)c.n_embd * 4; break;
        case BH_OP_ATTN: break;
        default: rows = c.n_vocab; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
    }
    if (bytes_per_launch)
        *bytes_per_launch = op == BH_OP_ATTN
                                // q, k, v in; K/V of positions 0..pos (fp32) read; the output written
                                ? (qd + 2 * kvd) * 4 + 2 * (int64_t)c.n_ctx * kvd * 4 + qd * 4
                                : rows * (k / bh::QK) * bh::Q4K_BYTES + xin + rows * 4;
    const int per_rep = op == BH_OP_LMHEAD ? 1 : c.n_layer;
    int rc = enqueue_op(st, op);  // warm-up
    if (rc != BH_OK) return rc;
    cudaEvent_t e0, e1;
    if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) return BH_EIO;
    cudaEventRecord(e0, st->stream);
    for (int r = 0; r < reps && rc == BH_OK; ++r) rc = enqueue_op(st, op);
    cudaEventRecord(e1, st->stream);
    float ms = 0.f;
    if (rc == BH_OK && (cudaEventSynchronize(e1) != cudaSuccess || cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess))
        rc = BH_EIO;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *avg_ms = ms / (float)(reps * per_rep);
    return rc;
}

int bh_stack_tensor(bh_stack* st, int layer, int which, void** ptr, int64_t* rows, int64_t* cols) {
    if (!st || !ptr) return BH_EINVAL;
    const bh_stack_config& c = st->cfg;
    int64_t r = 0, k = 0;
    if (which >= 0 && which < BH_W_PER_LAYER) {
        if (layer < 0 || layer >= c.n_layer) return BH_EINVAL;
        mat_dims(c, which, &r, &k);
        *ptr = const_cast<uint8_t*>(st->wq[(size_t)layer * BH_W_PER_LAYER + which]);
    } else if (which == BH_W_OUTPUT) {
        mat_dims(c, -1, &r, &k);
        *ptr = const_cast<uint8_t*>(st->wq[(size_t)c.n_layer * BH_W_PER_LAYER]);
    } else {
        const bool per_layer = which == BH_T_ATTN_NORM || which == BH_T_FFN_NORM || which == BH_T_Q_NORM ||
                               which == BH_T_K_NORM || which == BH_T_K_CACHE || which == BH_T_V_CACHE;
        if (per_layer && (layer < 0 || layer >= c.n_layer)) return BH_EINVAL;
        const int64_t kvd = (int64_t)c.n_head_kv * c.head_dim;
        switch (which) {
            case BH_T_ATTN_NORM: *ptr = st->attn_norm + (size_t)layer * c.n_embd; r = 1; k = c.n_embd; break;
            case BH_T_FFN_NORM: *ptr = st->ffn_norm + (size_t)layer * c.n_embd; r = 1; k = c.n_embd; break;
            case BH_T_Q_NORM: *ptr = st->q_norm + (size_t)layer * c.head_dim; r = 1; k = c.head_dim; break;
            case BH_T_K_NORM: *ptr = st->k_norm + (size_t)layer * c.head_dim; r = 1; k = c.head_dim; break;
            case BH_T_OUT_NORM: *ptr = st->out_norm; r = 1; k = c.n_embd; break;
            case BH_T_K_CACHE: *ptr = st->kc + (size_t)layer * c.n_ctx * kvd; r = c.n_ctx; k = kvd; break;
            case BH_T_V_CACHE: *ptr = st->vc + (size_t)layer * c.n_ctx * kvd; r = c.n_ctx; k = kvd; break;
            case BH_T_LOGITS: *ptr = st->logits; r = 1; k = c.n_vocab; break;
            case BH_T_HIDDEN: *ptr = st->h; r = 1; k = c.n_embd; break;
            default: return BH_EINVAL;
        }
    }
    if (rows) *rows = r;
    if (cols) *cols = k;
    return BH_OK;
}

}  // extern "C"
