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

#include <cooperative_groups.h>

#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"
#include "bh_math.cuh"

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
// attention for one decode token
// ---------------------------------------------------------------------------
struct AttnParams {
    const float* qkv;        // [q_dim | kv_dim | kv_dim]
    float* kc;               // K cache [n_ctx][n_head_kv][head_dim]
    float* vc;               // V cache
    const float* q_norm;     // [head_dim]
    const float* k_norm;     // [head_dim]
    const int* pos;          // device scalar: position of this token (set before the step)
    const float2* rope;      // [n_ctx][head_dim / 2]: (cos, sin) of every rotation angle
    float* out;              // [q_dim]
    int n_head, n_head_kv, head_dim, n_ctx;
    float eps;
    float qk_scale;          // 1.0f / sqrtf(head_dim), as the reference computes it
    int64_t* trace;          // timeline probe (builds with BH_TRACE only; else unused)
    const uint8_t* pf_ptr;   // L2 prefetch of the weights streamed next (null: none)
    int64_t pf_bytes;
    int* status;             // device status word (a bounded copy wait that ran out)
    TpLL ll;                 // row-split decode: out as exchanged pairs (ll.y_self set)
};

#ifdef BH_TRACE
// lane 0 of every warp records the global timer (ns) at point k
#define ATTN_TRACE_AT(k)                                                                                    \
    do {                                                                                                    \
        if (a.trace && (threadIdx.x & 31) == 0) {                                                           \
            uint64_t t_;                                                                                    \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                          \
            a.trace[((int64_t)blockIdx.x * DENSE_MAX_WARPS + (threadIdx.x >> 5)) * 8 + (k)] = (int64_t)t_; \
        }                                                                                                   \
    } while (0)
// each traced launch of a step writes its own region of the buffer
constexpr int64_t TRACE_LAUNCH = 256 * DENSE_MAX_WARPS * 8;
#else
#define ATTN_TRACE_AT(k) \
    do {                 \
    } while (0)
#endif

// Attention of one decode token, one CTA per query head, evaluated in the
// reference CPU backend's own order so that its output equals the engine's
// ggml graph (forward.cpp build_block_decode) bit for bit:
//  - per-head rms_norm (binary32 squares summed in double, 1/sqrtf(mean +
//    eps)) times the q / k norm weight;
//  - NeoX RoPE: x0' = x0 c - x1 s, x1' = x0 s + x1 c for the pairs (i, i + 64),
//    (c, s) from a table the host fills exactly as ggml's rope cache does
//    (theta = pos, theta *= powf(base, -2/n_dims) per pair, cosf / sinf);
//  - K.Q per position as ggml_vec_dot_f32's AVX2 path: one thread per
//    position keeps the 32 fma accumulators (the 4 x 8 vector accumulators;
//    accumulator l takes elements l, l + 32, l + 64, l + 96) and reduces them
//    in registers in GGML_F32x8_REDUCE's order; then ggml_scale (one multiply);
//  - soft_max: max, exp(x - max) by ggml_v_expf for every whole group of 8
//    (the n % 8 tail as (float)exp(double)), the per-8 float sums
//    ((p4+p0)+(p6+p2))+((p5+p1)+(p7+p3)) accumulated in double in group
//    order, then each p times (float)(1 / sum);
//  - V . p per dimension as ggml_vec_dot_f32 over the positions: thread d
//    keeps the 32 accumulators of positions t % 32 and reduces them in the
//    same order, the n % 32 tail added one by one in float.
// The new token's K (after RoPE) and V are appended at pos by the first head
// of each KV group; the other heads use their own copy of the same values for
// position pos and read only positions before it from the cache.
constexpr int ATTN_THREADS = 256;
constexpr int ATTN_WARPS = ATTN_THREADS / 32;
constexpr int ATTN_HD = 128;
// positions whose double sum of group partials is taken in order (beyond: a
// fixed tree, which differs from the reference's order only in the last bits
// of the double sum)
constexpr int ATTN_SEQ_GROUPS = 64;

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

// sum of the lane's 4 binary32 squares in double, then over the warp
__device__ __forceinline__ double warp_sumsq_d(float4 v) {
    double s = __dadd_rn(__dadd_rn((double)__fmul_rn(v.x, v.x), (double)__fmul_rn(v.y, v.y)),
                         __dadd_rn((double)__fmul_rn(v.z, v.z), (double)__fmul_rn(v.w, v.w)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    return s;
}

// rms_norm over head_dim = 128 values (4 per lane) then the norm weight:
// mean = (float)(sum / 128) (an exact power-of-two scaling), 1 / sqrtf(mean + eps)
__device__ __forceinline__ float4 head_rmsnorm(float4 x, float4 w, float eps) {
    const float mean = __double2float_rn(__dmul_rn(warp_sumsq_d(x), 1.0 / 128.0));
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
    return make_float4(__fmul_rn(__fmul_rn(x.x, r), w.x), __fmul_rn(__fmul_rn(x.y, r), w.y),
                       __fmul_rn(__fmul_rn(x.z, r), w.z), __fmul_rn(__fmul_rn(x.w, r), w.w));
}

// NeoX rotation of the 4 dims this lane holds (4l..4l+3); lanes l and l ^ 16
// hold the two halves of the same pairs; cs[j] = (cos, sin) of pair (4l + j) mod 64
__device__ __forceinline__ float rope1(float own, float other, float2 cs, bool low) {
    return low ? __fsub_rn(__fmul_rn(own, cs.x), __fmul_rn(other, cs.y))    // x0 c - x1 s
               : __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(own, cs.x));   // x0 s + x1 c
}
__device__ __forceinline__ float4 rope4(float4 x, const float2 (&cs)[4], bool low) {
    const float4 p = make_float4(__shfl_xor_sync(0xffffffffu, x.x, 16), __shfl_xor_sync(0xffffffffu, x.y, 16),
                                 __shfl_xor_sync(0xffffffffu, x.z, 16), __shfl_xor_sync(0xffffffffu, x.w, 16));
    return make_float4(rope1(x.x, p.x, cs[0], low), rope1(x.y, p.y, cs[1], low), rope1(x.z, p.z, cs[2], low),
                       rope1(x.w, p.w, cs[3], low));
}

// K / V history of one head is staged through shared memory in tiles of
// ATTN_TILE positions by bulk copies (one 512-byte row each, this GPU's own
// memory, no multicast) completing on an mbarrier; the first tile is issued
// before the programmatic wait (cache rows before pos do not depend on the
// previous kernel) and waited for only when the scores need it. Rows are
// ATTN_KROW floats apart: 16-byte reads of consecutive rows by consecutive
// threads then fall in distinct bank groups.
constexpr int ATTN_TILE = 128;
constexpr int ATTN_KROW = ATTN_HD + 4;

// Issue the bulk copy of row r (0 <= r < nh) of the tile into dst; every
// thread of the CTA issues at most one copy per tile, so the copies go out
// together (issued by one lane per warp, the 256 copies of a 128-position
// tile took ~0.8 us more on B200).
__device__ __forceinline__ void issue_kv_row(float* dst, const float* base, int64_t row_stride, int t0, int nh,
                                             uint64_t* bar, int r, uint64_t pol) {
    if (r >= 0 && r < nh) bulk_g2s(dst + r * ATTN_KROW, base + (int64_t)(t0 + r) * row_stride, ATTN_HD * 4, bar, pol);
}

// Arm (thread 0) and issue one tile of K and V rows.
__device__ __forceinline__ void load_kv_tile(float* s_kt, float* s_vt, const float* kbase, const float* vbase,
                                             int64_t row_stride, int t0, int nh, uint64_t* bar_k, uint64_t* bar_v,
                                             bool want_k, bool want_v, int tid, uint64_t pol) {
    if (tid == 0) {
        if (want_k) mbar_arrive_expect_tx(bar_k, (uint32_t)(nh * ATTN_HD * 4));
        if (want_v) mbar_arrive_expect_tx(bar_v, (uint32_t)(nh * ATTN_HD * 4));
    }
    __syncthreads();
    // the barrier was armed for nh * 512 bytes; K rows by threads 0 .. nh - 1,
    // V rows by threads ATTN_TILE .. ATTN_TILE + nh - 1
    static_assert(ATTN_THREADS >= 2 * ATTN_TILE, "one copy per thread");
    if (want_k) issue_kv_row(s_kt, kbase, row_stride, t0, nh, bar_k, tid, pol);
    if (want_v) issue_kv_row(s_vt, vbase, row_stride, t0, nh, bar_v, tid - ATTN_TILE, pol);
}

template <bool LL>
__global__ void __launch_bounds__(ATTN_THREADS) attn_head_kernel(const AttnParams a) {
    extern __shared__ __align__(128) float smem_f[];
    float* s_kt = smem_f;                              // [ATTN_TILE][ATTN_KROW] K rows of the current tile
    float* s_vt = smem_f + ATTN_TILE * ATTN_KROW;      // [ATTN_TILE][ATTN_KROW] V rows
    float* s_p = smem_f + 2 * ATTN_TILE * ATTN_KROW;   // [n_ctx] scores, then probabilities
    __shared__ __align__(16) float s_q[ATTN_HD], s_k[ATTN_HD], s_v[ATTN_HD];
    __shared__ float s_red[ATTN_WARPS];
    __shared__ float s_gsum[ATTN_SEQ_GROUPS];
    __shared__ float s_inv;
    __shared__ __align__(8) uint64_t bar_k, bar_v;
    __shared__ int s_ok;
    constexpr int HD = ATTN_HD;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int group = a.n_head / a.n_head_kv, g = h / group;
    const int q_dim = a.n_head * HD, kv_dim = a.n_head_kv * HD;
    const int64_t row_stride = (int64_t)kv_dim;
    const float* kbase = a.kc + (int64_t)g * HD;
    const float* vbase = a.vc + (int64_t)g * HD;
    ATTN_TRACE_AT(0);

    // before the wait, nothing that depends on the previous kernel: the
    // copies of the first tile of the K / V history, then the norm weights
    // and the rotation table row of pos (pos is set before the step), whose
    // loads are left in flight over the wait
    const uint64_t keep = policy_evict_last();
    if (tid == 0) {
        mbar_init(&bar_k, 1);
        mbar_init(&bar_v, 1);
        fence_mbar_init();
        s_ok = 1;
    }
    const int pos = *a.pos;
    load_kv_tile(s_kt, s_vt, kbase, vbase, row_stride, 0, min(pos, ATTN_TILE), &bar_k, &bar_v, true, true, tid, keep);
    const int n = pos + 1;
    float4 qn = f4_zero(), kn = f4_zero();
    float2 cs[4];
    if (w == 0) {
        qn = ldg_f4_keep(a.q_norm + 4 * lane, keep);
        kn = ldg_f4_keep(a.k_norm + 4 * lane, keep);
        const float4* rt = reinterpret_cast<const float4*>(a.rope + (int64_t)pos * (HD / 2) + 4 * (lane & 15));
        const float4 r01 = rt[0], r23 = rt[1];
        cs[0] = make_float2(r01.x, r01.y); cs[1] = make_float2(r01.z, r01.w);
        cs[2] = make_float2(r23.x, r23.y); cs[3] = make_float2(r23.z, r23.w);
    }
    ATTN_TRACE_AT(4);
    uint32_t ph_k = 0, ph_v = 0;
    prefetch_share(a.pf_ptr, a.pf_bytes, (int64_t)blockIdx.x * ATTN_WARPS + w, (int64_t)gridDim.x * ATTN_WARPS, lane);
    pdl_trigger();
    ATTN_TRACE_AT(7);
    pdl_wait();
    ATTN_TRACE_AT(5);
    const uint32_t gen_out = LL ? tp_gen(a.ll, a.ll.gen_out) : 0u;

    // this head's q, the group's k and v of this token: norm, rotation
    if (w == 0) {
        const float4 q = reinterpret_cast<const float4*>(a.qkv + (int64_t)h * HD)[lane];
        const float4 k = reinterpret_cast<const float4*>(a.qkv + q_dim + (int64_t)g * HD)[lane];
        const float4 v = reinterpret_cast<const float4*>(a.qkv + q_dim + kv_dim + (int64_t)g * HD)[lane];
        const bool low = lane < 16;
        const float4 qr = rope4(head_rmsnorm(q, qn, a.eps), cs, low);
        const float4 kr = rope4(head_rmsnorm(k, kn, a.eps), cs, low);
        reinterpret_cast<float4*>(s_q)[lane] = qr;
        reinterpret_cast<float4*>(s_k)[lane] = kr;
        reinterpret_cast<float4*>(s_v)[lane] = v;
        if (h % group == 0) {
            reinterpret_cast<float4*>(a.kc + (int64_t)pos * row_stride + (int64_t)g * HD)[lane] = kr;
            reinterpret_cast<float4*>(a.vc + (int64_t)pos * row_stride + (int64_t)g * HD)[lane] = v;
        }
    }
    ATTN_TRACE_AT(1);

    // scores: thread r of a tile computes position t0 + r whole, in
    // ggml_vec_dot_f32's order (accumulator l = element l of the 4 x 8
    // vectors, fma over the 4 steps of 32), then GGML_F32x8_REDUCE in
    // registers and ggml_scale
    float tmax = -INFINITY;
    bool ok = true;
    for (int t0 = 0; t0 < n && ok; t0 += ATTN_TILE) {
        const int nt = min(ATTN_TILE, n - t0);
        if (t0 > 0) {
            __syncthreads();  // every thread is done with the previous K tile
            fence_proxy_async_smem();
            load_kv_tile(s_kt, s_vt, kbase, vbase, row_stride, t0, min(nt, pos - t0), &bar_k, &bar_v, true, false,
                         tid, keep);
        }
        // one decision for the whole block (and s_q / s_k of warp 0 visible)
        ok = __syncthreads_and(mbar_wait_bounded(&bar_k, ph_k)) != 0;
        if (!ok) break;
        ph_k ^= 1u;
        for (int r = tid; r < nt; r += ATTN_THREADS) {
            const int t = t0 + r;
            const float4* krow = reinterpret_cast<const float4*>(t == pos ? s_k : s_kt + r * ATTN_KROW);
            const float4* qv = reinterpret_cast<const float4*>(s_q);
            float acc[32];
#pragma unroll
            for (int l = 0; l < 32; ++l) acc[l] = 0.f;
#pragma unroll
            for (int i0 = 0; i0 < 4; ++i0) {
#pragma unroll
                for (int l4 = 0; l4 < 8; ++l4) {
                    const float4 kx = krow[8 * i0 + l4], qx = qv[8 * i0 + l4];
                    acc[4 * l4 + 0] = __fmaf_rn(kx.x, qx.x, acc[4 * l4 + 0]);
                    acc[4 * l4 + 1] = __fmaf_rn(kx.y, qx.y, acc[4 * l4 + 1]);
                    acc[4 * l4 + 2] = __fmaf_rn(kx.z, qx.z, acc[4 * l4 + 2]);
                    acc[4 * l4 + 3] = __fmaf_rn(kx.w, qx.w, acc[4 * l4 + 3]);
                }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                acc[e] = __fadd_rn(acc[e], acc[16 + e]);
                acc[8 + e] = __fadd_rn(acc[8 + e], acc[24 + e]);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], acc[8 + e]);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = __fadd_rn(acc[e], acc[e + 4]);
            const float sc = __fmul_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])), a.qk_scale);
            s_p[t] = sc;
            tmax = fmaxf(tmax, sc);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    if (lane == 0) s_red[w] = tmax;
    if (!ok && tid == 0) s_ok = 0;
    __syncthreads();
    ATTN_TRACE_AT(2);
    if (!s_ok) {
        // a copy wait ran out: report, give the copies in flight (the K tile
        // waited for, the first V tile) a second bounded wait, write no output
        if (tid == 0) {
            set_status(a.status, ST_TIMEOUT);
            mbar_wait_bounded(&bar_k, ph_k);
            mbar_wait_bounded(&bar_v, ph_v);
        }
        return;
    }
    float mx = s_red[0];
#pragma unroll
    for (int i = 1; i < ATTN_WARPS; ++i) mx = fmaxf(mx, s_red[i]);

    // soft_max: p = exp(s - max); group sums of 8 in float; their double sum
    const int n8 = n & ~7, ng = n8 >> 3;
    for (int t = tid; t < n; t += ATTN_THREADS) {
        const float x = __fsub_rn(s_p[t], mx);
        s_p[t] = t < n8 ? exp_ggml(x) : __double2float_rn(exp((double)x));
    }
    __syncthreads();
    for (int gi = tid; gi < ng && gi < ATTN_SEQ_GROUPS; gi += ATTN_THREADS) {
        const float* v = s_p + 8 * gi;
        s_gsum[gi] = __fadd_rn(__fadd_rn(__fadd_rn(v[4], v[0]), __fadd_rn(v[6], v[2])),
                               __fadd_rn(__fadd_rn(v[5], v[1]), __fadd_rn(v[7], v[3])));
    }
    __syncthreads();
    if (w == 0) {
        double sum = 0.0;
        if (ng <= ATTN_SEQ_GROUPS) {
            if (lane == 0)
                for (int gi = 0; gi < ng; ++gi) sum = __dadd_rn(sum, (double)s_gsum[gi]);
        } else {
            for (int gi = lane; gi < ng; gi += 32) {
                const float* v = s_p + 8 * gi;
                const float gs = __fadd_rn(__fadd_rn(__fadd_rn(v[4], v[0]), __fadd_rn(v[6], v[2])),
                                           __fadd_rn(__fadd_rn(v[5], v[1]), __fadd_rn(v[7], v[3])));
                sum = __dadd_rn(sum, (double)gs);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
        }
        if (lane == 0) {
            for (int t = n8; t < n; ++t) sum = __dadd_rn(sum, (double)s_p[t]);
            s_inv = __double2float_rn(__ddiv_rn(1.0, sum));
        }
    }
    __syncthreads();
    const float inv = s_inv;
    for (int t = tid; t < n; t += ATTN_THREADS) s_p[t] = __fmul_rn(s_p[t], inv);
    __syncthreads();
    ATTN_TRACE_AT(3);

    // out[d] = V[.][d] . p: thread d keeps the 32 accumulators of positions
    // t mod 32, chunk after chunk, from the staged V tiles
    const int d = tid;
    const int np = n & ~31;
    float acc[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) acc[r] = 0.f;
    float sumf = 0.f;
    for (int t0 = 0; t0 < n; t0 += ATTN_TILE) {
        const int nt = min(ATTN_TILE, n - t0);
        if (t0 > 0) {
            __syncthreads();
            fence_proxy_async_smem();
            load_kv_tile(s_kt, s_vt, kbase, vbase, row_stride, t0, min(nt, pos - t0), &bar_k, &bar_v, false, true,
                         tid, keep);
        }
        if (!__syncthreads_and(mbar_wait_bounded(&bar_v, ph_v))) {
            if (tid == 0) {
                set_status(a.status, ST_TIMEOUT);
                mbar_wait_bounded(&bar_v, ph_v);  // (this tile's copies are the last in flight)
            }
            return;
        }
        ph_v ^= 1u;
        if (d < HD) {
            const int cend = min(np, t0 + nt);
            for (int c0 = t0; c0 < cend; c0 += 32) {
#pragma unroll
                for (int r = 0; r < 32; ++r) {
                    const int t = c0 + r;
                    const float v = t == pos ? s_v[d] : s_vt[(t - t0) * ATTN_KROW + d];
                    acc[r] = __fmaf_rn(v, s_p[t], acc[r]);
                }
            }
            if (t0 + nt >= n) {
                // GGML_F32x8_REDUCE: accumulator j element e is acc[8 j + e]
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    acc[e] = __fadd_rn(acc[e], acc[16 + e]);
                    acc[8 + e] = __fadd_rn(acc[8 + e], acc[24 + e]);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], acc[8 + e]);
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[e] = __fadd_rn(acc[e], acc[e + 4]);
                sumf = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
            }
            // the n % 32 tail, one by one in float (its rows are in this tile)
            for (int t = max(np, t0); t < t0 + nt; ++t) {
                const float v = t == pos ? s_v[d] : s_vt[(t - t0) * ATTN_KROW + d];
                sumf = __fadd_rn(sumf, __fmul_rn(v, s_p[t]));
            }
        }
    }
    if (d < HD) {
        if (LL)
            tp_store(a.ll, (int64_t)h * HD + d, sumf, gen_out);
        else
            a.out[(int64_t)h * HD + d] = sumf;
    }
    ATTN_TRACE_AT(6);
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
    float2* rope;                   // [n_ctx][head_dim / 2] (cos, sin) of the rotation angles
    float *kc, *vc;
    float *x_in, *h, *qkv, *attn, *gu, *logits, *cand_val;
    float *cap_h_attn, *cap_gate_up;  // the last layer's h after O + residual, its gate | up rows
    int32_t *cand_idx, *tok;
    int* pos;
    int32_t* host_tok = nullptr;    // pinned
    float* host_x = nullptr;        // pinned staging for the host-buffer call
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int lm_grid = 0;
    int64_t step_bytes = 0;         // algorithmic bytes of one decode step (this GPU's rows)
    int64_t launches = 0;           // kernel launches in one step
    // Row split over tp_world GPUs (1: the whole model here). This rank owns
    // query heads [qh0, qh0 + n_head_l), KV heads [kh0, kh0 + n_head_kv_l),
    // rows [e0, e0 + n_embd_l) of O and down, [f0, f0 + n_ff_l) of gate and
    // up, [v0, v0 + n_vocab_l) of the LM head.
    int tp_rank = 0, tp_world = 1;
    int qh0 = 0, kh0 = 0, n_head_l = 0, n_head_kv_l = 0;
    int64_t e0 = 0, f0 = 0, v0 = 0, n_embd_l = 0, n_ff_l = 0, n_vocab_l = 0;
    // exchange region (one allocation, exported to the peers through CUDA
    // IPC): the full h, attention output and SwiGLU output vectors, the step
    // counter and the LM head's pick mailbox
    uint8_t* xbuf = nullptr;
    size_t xbytes = 0, x_h = 0, x_attn = 0, x_gu = 0, x_step = 0, x_box = 0;
    uint8_t* peer_x[bh::TP_MAX_WORLD] = {};  // every rank's exchange region as mapped here (own at [tp_rank])
    bool tp_connected = false;
};

namespace {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Exchanges of one layer in the row-split step (generation offsets): the
// attention output, h after O, the SwiGLU output, h after down.
constexpr int XG_ATTN = 0, XG_H_O = 1, XG_GU = 2, XG_H_DOWN = 3, XG_PER_LAYER = 4;

int check_cfg(const bh_stack_config* c) {
    if (!c) return BH_EINVAL;
    if (c->n_layer < 1 || c->n_embd < 256 || c->n_embd % 256 || c->n_ff < 256 || c->n_ff % 256) return BH_EINVAL;
    if (c->head_dim != bh::ATTN_HD) return BH_EINVAL;  // the attention kernel is written for 128
    if (c->n_head < 1 || c->n_head_kv < 1 || c->n_head % c->n_head_kv) return BH_EINVAL;
    if ((c->n_head * c->head_dim) % 256 || c->n_vocab < 1 || c->n_ctx < 1 || c->n_ctx > 8192) return BH_EINVAL;
    return BH_OK;
}

// Rows of matrix `which` (-1: the LM head) this rank holds, the model row
// the first of them is, and the columns.
void mat_dims(const bh_stack* st, int which, int64_t* rows, int64_t* cols, int64_t* row0 = nullptr) {
    const bh_stack_config& c = st->cfg;
    const int64_t hd = c.head_dim, qd = (int64_t)c.n_head * hd;
    int64_t r0 = 0;
    switch (which) {
        case BH_W_Q: *rows = st->n_head_l * hd; r0 = st->qh0 * hd; *cols = c.n_embd; break;
        case BH_W_K:
        case BH_W_V: *rows = st->n_head_kv_l * hd; r0 = st->kh0 * hd; *cols = c.n_embd; break;
        case BH_W_O: *rows = st->n_embd_l; r0 = st->e0; *cols = qd; break;
        case BH_W_GATE:
        case BH_W_UP: *rows = st->n_ff_l; r0 = st->f0; *cols = c.n_embd; break;
        case BH_W_DOWN: *rows = st->n_embd_l; r0 = st->e0; *cols = c.n_ff; break;
        default: *rows = st->n_vocab_l; r0 = st->v0; *cols = c.n_embd; break;  // LM head
    }
    if (row0) *row0 = r0;
}

// Exchanged-pair parameters of a launch on a row split (world 1: none):
// input = the pairs of exchange (l_in, xg_in) at byte offset in_off of the
// exchange region (xg_in < 0: the plain fp32 input), output = exchange
// (l_out, xg_out) into the pairs at byte offset out_off of every rank's
// region (xg_out < 0: the plain output).
bh::TpLL tp_ll(const bh_stack* st, size_t in_off, int l_in, int xg_in, size_t out_off, int l_out, int xg_out) {
    bh::TpLL ll{};
    if (st->tp_world < 2) return ll;
    ll.step = reinterpret_cast<const uint32_t*>(st->xbuf + st->x_step);
    ll.gen_mul = (uint32_t)(st->cfg.n_layer * XG_PER_LAYER);
    if (xg_in >= 0) {
        ll.x = reinterpret_cast<const uint64_t*>(st->xbuf + in_off);
        ll.gen_in = (uint32_t)(l_in * XG_PER_LAYER + xg_in + 1);
    }
    if (xg_out >= 0) {
        ll.y_self = reinterpret_cast<uint64_t*>(st->xbuf + out_off);
        for (int q = 0; q < st->tp_world; ++q)
            if (q != st->tp_rank) ll.y_peer[ll.npeer++] = reinterpret_cast<uint64_t*>(st->peer_x[q] + out_off);
        ll.gen_out = (uint32_t)(l_out * XG_PER_LAYER + xg_out + 1);
    }
    return ll;
}

uint64_t tensor_seed(uint64_t seed, int layer, int which) {
    uint64_t z = seed ^ (0x51ed2701a3b4c5d6ULL + (uint64_t)layer * 0x9e3779b97f4a7c15ULL + (uint64_t)which * 0xd6e8feb86659fd93ULL);
    z = (z ^ (z >> 31)) * 0x7fb5d329728ea185ULL;
    return z ^ (z >> 27);
}

// Layer l's gate / up launch: the two matrices as the segments of one row-pair
// launch; st->gu receives silu(gate) * up (n_ff values).
bh::MatvecParams gate_up_params(bh_stack* st, int l) {
    const bh_stack_config& c = st->cfg;
    const uint8_t* const* W = st->wq + (size_t)l * BH_W_PER_LAYER;
    const int64_t nf = st->n_ff_l;  // this rank's rows of gate and of up (all of them on one GPU)
    bh::MatvecParams p = bh::base_params(st->ctx, W[BH_W_GATE], 2 * nf, c.n_embd, 1, st->gu + st->f0);
    p.w[1] = p.w[2] = W[BH_W_UP];
    p.seg_end[0] = nf;
    p.seg_end[1] = p.seg_end[2] = 2 * nf;
    p.ldy = c.n_ff;
    p.xf = st->h;
    p.gamma = st->ffn_norm + (size_t)l * c.n_embd;
    p.eps = c.rms_eps;
    return p;
}

// The weights are one allocation in streaming order (per layer Q K V O gate
// up down, then the LM head): a launch whose own weights end at `end`
// prefetches the next prefetch_bytes of that order into the L2 (after the LM
// head, the next step's first layer).
void set_prefetch(const bh_stack* st, const uint8_t* end, const uint8_t** ptr, int64_t* bytes) {
    const int64_t win = st->plan.prefetch_bytes;
    *ptr = nullptr;
    *bytes = 0;
    if (win <= 0) return;
    int64_t off = end - st->wbuf;
    if (off >= (int64_t)st->wbytes) off = 0;
    const int64_t left = (int64_t)st->wbytes - off;
    *ptr = st->wbuf + off;
    *bytes = (win < left ? win : left) & ~(int64_t)15;
}

// End of matrix i of the weight allocation.
const uint8_t* mat_end(const bh_stack* st, int i) {
    const bh_stack_config& c = st->cfg;
    int64_t r, k;
    mat_dims(st, i < c.n_layer * BH_W_PER_LAYER ? i % BH_W_PER_LAYER : -1, &r, &k);
    return st->wq[i] + r * (k / bh::QK) * bh::Q4K_BYTES;
}

int stack_matvec(bh_stack* st, bh::MatvecParams& p, int src, int epi, bool pdl) {
#ifdef BH_TRACE
    if (st->ctx->trace) p.trace = st->ctx->trace + st->launches * bh::TRACE_LAUNCH;
#endif
    return bh::run_matvec(&st->plan, p, BH_FOLD_X86, src, epi, st->stream, pdl);
}

// Attention of layer l over positions 0..pos (one CTA per query head).
// (Row split: this rank's query heads and their KV heads, the output at the
// heads' place in the full vector, also stored into the peers' copies.)
int launch_attn(bh_stack* st, int l, bool pdl) {
    const bh_stack_config& c = st->cfg;
    const int64_t kvd = (int64_t)st->n_head_kv_l * c.head_dim;
    bh::AttnParams a{};
    a.qkv = st->qkv;
    a.kc = st->kc + (size_t)l * c.n_ctx * kvd;
    a.vc = st->vc + (size_t)l * c.n_ctx * kvd;
    a.q_norm = st->q_norm + (size_t)l * c.head_dim;
    a.k_norm = st->k_norm + (size_t)l * c.head_dim;
    a.pos = st->pos;
    a.rope = st->rope;
    a.out = st->attn + (size_t)st->qh0 * c.head_dim;
    a.ll = tp_ll(st, 0, 0, -1, st->x_attn + 8 * (size_t)st->qh0 * c.head_dim, l, XG_ATTN);
    a.n_head = st->n_head_l;
    a.n_head_kv = st->n_head_kv_l;
    a.head_dim = c.head_dim;
    a.n_ctx = c.n_ctx;
    a.eps = c.rms_eps;
    a.qk_scale = 1.0f / std::sqrt((float)c.head_dim);  // forward.cpp: 1.0f / sqrtf((float)head_dim)
    a.status = st->ctx->d_status;
    set_prefetch(st, mat_end(st, l * BH_W_PER_LAYER + BH_W_V), &a.pf_ptr, &a.pf_bytes);
    a.trace = nullptr;
#ifdef BH_TRACE
    if (st->ctx->trace) a.trace = st->ctx->trace + st->launches * bh::TRACE_LAUNCH;
#endif
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)st->n_head_l);
    cfg.blockDim = dim3((unsigned)bh::ATTN_THREADS);
    cfg.dynamicSmemBytes = sizeof(float) * ((size_t)2 * bh::ATTN_TILE * bh::ATTN_KROW + (size_t)c.n_ctx);
    cfg.stream = st->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    // (the row split's variant stores the output as exchanged pairs)
    auto kern = a.ll.y_self ? bh::attn_head_kernel<true> : bh::attn_head_kernel<false>;
    static std::atomic<uint64_t> attr_devices[2];
    // the same shared-memory carveout as the matvecs around it
    if (!bh::attrs_on_device(attr_devices[a.ll.y_self ? 1 : 0], [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
                       cudaSuccess &&
                   cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared) == cudaSuccess;
        }))
        return BH_EIO;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? BH_OK : BH_EIO;
}

// Enqueue one decode step on st->stream (captured into the graph). On a row
// split every launch works this rank's rows; the vectors the next launch
// reads whole (attention output, h, SwiGLU output) are exchanged as
// generation-tagged pairs that the producing launch stores into every rank's
// copy and the reading launch polls for.
int enqueue_step(bh_stack* st) {
    const bh_stack_config& c = st->cfg;
    bh_ctx* ctx = st->ctx;
    const int64_t hd = c.head_dim, qd = (int64_t)c.n_head * hd;
    const int64_t qd_l = (int64_t)st->n_head_l * hd, kvd_l = (int64_t)st->n_head_kv_l * hd;
    const bool tp = st->tp_world > 1;
    int rc;
    const cudaError_t ce =
        tp ? cudaMemcpy2DAsync(st->xbuf + st->x_h, 8, st->x_in, 4, 4, (size_t)c.n_embd, cudaMemcpyDeviceToDevice,
                               st->stream)  // the values of h's pairs (the first QKV reads x_in itself)
           : cudaMemcpyAsync(st->h, st->x_in, sizeof(float) * c.n_embd, cudaMemcpyDeviceToDevice, st->stream);
    if (ce != cudaSuccess) return BH_EIO;
    st->step_bytes = 0;
    st->launches = 0;
    auto account = [&](const bh::MatvecParams& p, int b_in_bytes, int64_t out_rows) {
        st->step_bytes += p.N * (int64_t)p.nb * bh::Q4K_BYTES + b_in_bytes + out_rows * 4;
        st->launches += 1;
    };
    const size_t h_e0 = st->x_h + 8 * (size_t)st->e0, gu_f0 = st->x_gu + 8 * (size_t)st->f0;
    for (int l = 0; l < c.n_layer; ++l) {
        const uint8_t* const* W = st->wq + (size_t)l * BH_W_PER_LAYER;
        const bool last = l == c.n_layer - 1;
        // 1. QKV (this rank's heads of the whole h)
        bh::MatvecParams p = bh::base_params(ctx, W[BH_W_Q], qd_l + 2 * kvd_l, c.n_embd, 1, st->qkv);
        p.w[1] = W[BH_W_K];
        p.w[2] = W[BH_W_V];
        p.seg_end[0] = qd_l;
        p.seg_end[1] = qd_l + kvd_l;
        p.seg_end[2] = qd_l + 2 * kvd_l;
        p.xf = tp && l == 0 ? st->x_in : st->h;
        p.gamma = st->attn_norm + (size_t)l * c.n_embd;
        p.eps = c.rms_eps;
        p.ll = tp_ll(st, st->x_h, l - 1, l > 0 ? XG_H_DOWN : -1, 0, 0, -1);
        set_prefetch(st, mat_end(st, l * BH_W_PER_LAYER + BH_W_V), &p.pf_ptr, &p.pf_bytes);
        if ((rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, l > 0)) != BH_OK) return rc;
        account(p, c.n_embd * 4, p.N);
        // 2. attention
        if ((rc = launch_attn(st, l, true)) != BH_OK) return rc;
        st->launches += 1;
        // 3. O projection, residual add on this rank's rows of h
        p = bh::base_params(ctx, W[BH_W_O], st->n_embd_l, qd, 1, st->h + st->e0);
        p.xf = st->attn;
        if (last && !tp) p.capture = st->cap_h_attn;
        p.ll = tp_ll(st, st->x_attn, l, XG_ATTN, h_e0, l, XG_H_O);
        set_prefetch(st, mat_end(st, l * BH_W_PER_LAYER + BH_W_O), &p.pf_ptr, &p.pf_bytes);
        if ((rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, true)) != BH_OK) return rc;
        account(p, (int)qd * 4, p.N);
        // 4. gate / up in row pairs, silu(gate) * up in the epilogue
        p = gate_up_params(st, l);
        if (last && !tp) p.capture = st->cap_gate_up;
        p.ll = tp_ll(st, st->x_h, l, XG_H_O, gu_f0, l, XG_GU);
        set_prefetch(st, mat_end(st, l * BH_W_PER_LAYER + BH_W_UP), &p.pf_ptr, &p.pf_bytes);
        if ((rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_SWIGLU, true)) != BH_OK) return rc;
        account(p, c.n_embd * 4, st->n_ff_l);
        // 5. down, residual add on this rank's rows of h
        p = bh::base_params(ctx, W[BH_W_DOWN], st->n_embd_l, c.n_ff, 1, st->h + st->e0);
        p.xf = st->gu;
        p.ll = tp_ll(st, st->x_gu, l, XG_GU, h_e0, l, XG_H_DOWN);
        set_prefetch(st, mat_end(st, l * BH_W_PER_LAYER + BH_W_DOWN), &p.pf_ptr, &p.pf_bytes);
        if ((rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, true)) != BH_OK) return rc;
        account(p, c.n_ff * 4, p.N);
    }
    // LM head + argmax (row split: this rank's vocabulary rows, then the pick
    // merged across ranks through the mailboxes)
    bh::MatvecParams p = bh::base_params(ctx, st->wq[(size_t)c.n_layer * BH_W_PER_LAYER], st->n_vocab_l, c.n_embd, 1,
                                         st->logits);
    p.xf = st->h;
    p.gamma = st->out_norm;
    p.eps = c.rms_eps;
    p.cand_val = st->cand_val;
    p.cand_idx = st->cand_idx;
    p.ll = tp_ll(st, st->x_h, c.n_layer - 1, XG_H_DOWN, 0, 0, -1);
    set_prefetch(st, mat_end(st, c.n_layer * BH_W_PER_LAYER), &p.pf_ptr, &p.pf_bytes);
#ifdef BH_TRACE
    if (ctx->trace) p.trace = ctx->trace + st->launches * bh::TRACE_LAUNCH;
#endif
    const int grid = bh::plan_for(ctx, p, 0, BH_FOLD_X86);
    if (grid < 0) return grid;
    st->lm_grid = grid;
    bh::LaunchOpts o;
    o.stream = st->stream;
    o.grid = grid;
    o.pdl = true;
    if ((rc = bh::launch_matvec(p, BH_FOLD_X86, bh::ACT_F32_RMSNORM, bh::EPI_ARGMAX, o)) != BH_OK) return rc;
    account(p, c.n_embd * 4, p.N);
    if (tp) {
        void* boxes[bh::TP_MAX_WORLD];
        for (int q = 0; q < st->tp_world; ++q) boxes[q] = st->peer_x[q] + st->x_box;
        uint32_t* step = reinterpret_cast<uint32_t*>(st->xbuf + st->x_step);
        rc = bh::launch_xchg_argmax(st->cand_val, st->cand_idx, grid, 1, st->v0, st->tp_rank, st->tp_world, boxes, 0,
                                    st->tok, nullptr, ctx->d_status, st->stream, step, step);
    } else {
        rc = bh::launch_argmax_finish(st->cand_val, st->cand_idx, grid, 1, st->tok, nullptr, st->stream, true);
    }
    if (rc != BH_OK) return rc;
    st->launches += 1;
    return BH_OK;
}

// Launch one op of the step for every layer (or the LM head once), eagerly,
// with the same parameters the step uses, the layer launches programmatic as
// in the step.
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
        const int grid = bh::plan_for(ctx, p, 0, BH_FOLD_X86);
        if (grid < 0) return grid;
        bh::LaunchOpts o;
        o.stream = st->stream;
        o.grid = grid;
        return bh::launch_matvec(p, BH_FOLD_X86, bh::ACT_F32_RMSNORM, bh::EPI_ARGMAX, o);
    }
    if (op == BH_OP_ATTN) {
        for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) rc = launch_attn(st, l, true);
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
                rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_STORE, true);
                break;
            case BH_OP_O:
                p = bh::base_params(ctx, W[BH_W_O], c.n_embd, qd, 1, st->h);
                p.xf = st->attn;
                rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, true);
                break;
            case BH_OP_GATE_UP:
                p = gate_up_params(st, l);
                rc = stack_matvec(st, p, bh::ACT_F32_RMSNORM, bh::EPI_SWIGLU, true);
                break;
            case BH_OP_DOWN:
                p = bh::base_params(ctx, W[BH_W_DOWN], c.n_embd, c.n_ff, 1, st->h);
                p.xf = st->gu;
                rc = stack_matvec(st, p, bh::ACT_F32, bh::EPI_ADD, true);
                break;
            default:
                return BH_EINVAL;
        }
    }
    return rc;
}

int ensure_graph(bh_stack* st) {
    if (st->exec) return BH_OK;
    if (st->tp_world > 1 && !st->tp_connected) return BH_EINVAL;  // bh_stack_tp_connect first
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
    return bh_stack_create_tp(ctx, cfg, seed, 0, 1, out);
}

int bh_stack_create_tp(bh_ctx* ctx, const bh_stack_config* cfg, uint64_t seed, int rank, int world, bh_stack** out) {
    if (!ctx || !out) return BH_EINVAL;
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc != BH_OK) return rc;
    // a row split keeps whole KV groups (and so whole query heads) on one
    // rank, and 8-row multiples of every split matrix
    if (world < 1 || world > bh::TP_MAX_WORLD || rank < 0 || rank >= world || cfg->n_head_kv % world ||
        cfg->n_embd % (8 * world) || cfg->n_ff % (8 * world) || cfg->n_vocab < world)
        return BH_EINVAL;
    // (a split's launches read the exchanged vectors in their one-round
    // staging: at most 32 blocks through RMSNorm, 48 plain)
    if (world > 1 && (cfg->n_embd > 32 * bh::QK || (int64_t)cfg->n_head * cfg->head_dim > 48 * bh::QK ||
                      cfg->n_ff > 48 * bh::QK))
        return BH_EINVAL;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return BH_ENODEV;
    bh_stack* st = new (std::nothrow) bh_stack();
    if (!st) return BH_ENOMEM;
    st->ctx = ctx;
    st->tp_rank = rank;
    st->tp_world = world;
    st->n_head_l = cfg->n_head / world;
    st->qh0 = st->n_head_l * rank;
    st->n_head_kv_l = cfg->n_head_kv / world;
    st->kh0 = st->n_head_kv_l * rank;
    st->n_embd_l = cfg->n_embd / world;
    st->e0 = st->n_embd_l * rank;
    st->n_ff_l = cfg->n_ff / world;
    st->f0 = st->n_ff_l * rank;
    st->v0 = (int64_t)cfg->n_vocab * rank / world;  // the LM head's rows: an even split, the last shards may differ by one
    st->n_vocab_l = (int64_t)cfg->n_vocab * (rank + 1) / world - st->v0;
    // Launch plan of the layer matvecs, unless the caller tuned a per-SM
    // budget on ctx: at most 168 KiB of shared memory per SM, 1440-byte row
    // slices per stage (one 16-warp CTA per SM; the planner picks the threads
    // per row), and one ring stage per warp issued before the programmatic
    // wait, the rest right after the activation loads (measured on B200:
    // 1.557 ms per token against 1.575 with 1152-byte slices, 1.567 with
    // 1728, 1.79-1.87 with 864 or 576; the whole ring before the wait cost
    // ~0.02 ms). The LM head keeps ctx's plan.
    st->plan = *ctx;
    if (ctx->sm_budget == 0) {
        st->plan.sm_budget = 168 * 1024;
        st->plan.stage_bytes = 1440;
        st->plan.tpr_narrow = 8;
        st->plan.prefill_stages = 1;
    }
    // L2 prefetch of the weights ahead measured no faster on B200 (16 MiB:
    // -2%; 48-96 MiB: +9% to +39% per token): off unless tuned
    if (ctx->prefetch_bytes < 0) st->plan.prefetch_bytes = 0;
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
        mat_dims(st, i < c.n_layer * BH_W_PER_LAYER ? i % BH_W_PER_LAYER : -1, &r, &k);
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
    // fp32 side buffers (this rank's heads and rows)
    const int64_t qd = (int64_t)c.n_head * c.head_dim;
    const int64_t qd_l = (int64_t)st->n_head_l * c.head_dim, kvd = (int64_t)st->n_head_kv_l * c.head_dim;
    const int cand_max = ctx->num_sms * 4;
    size_t fl = 0;
    auto take = [&](int64_t n) { const size_t o = fl; fl = align_up(fl + (size_t)n, 64); return o; };
    const size_t o_an = take((int64_t)c.n_layer * c.n_embd), o_fn = take((int64_t)c.n_layer * c.n_embd);
    const size_t o_qn = take((int64_t)c.n_layer * c.head_dim), o_kn = take((int64_t)c.n_layer * c.head_dim);
    const size_t o_on = take(c.n_embd);
    const size_t o_kc = take((int64_t)c.n_layer * c.n_ctx * kvd), o_vc = take((int64_t)c.n_layer * c.n_ctx * kvd);
    const size_t o_x = take(c.n_embd), o_qkv = take(qd_l + 2 * kvd);
    const size_t o_lg = take(st->n_vocab_l), o_cv = take(cand_max);
    const size_t o_ci = take(cand_max), o_tk = take(1), o_ps = take(1);
    const size_t o_rf = take((int64_t)c.n_ctx * c.head_dim);  // (cos, sin) per position and pair
    const size_t o_ch = take(c.n_embd), o_cg = take(2 * (int64_t)c.n_ff);
    // the exchange region: h, attention output, SwiGLU output (whole
    // vectors), the step counter, the pick mailbox
    size_t xl = 0;
    auto xtake = [&](size_t bytes) { const size_t o = xl; xl = align_up(xl + bytes, 256); return o; };
    st->x_h = xtake(sizeof(uint64_t) * (size_t)c.n_embd);  // fp32 values on one GPU, (value, generation) pairs on a split
    st->x_attn = xtake(sizeof(uint64_t) * (size_t)qd);
    st->x_gu = xtake(sizeof(uint64_t) * (size_t)c.n_ff);
    st->x_step = xtake(sizeof(uint32_t));
    st->x_box = xtake(bh_xchg_mailbox_bytes());
    st->xbytes = xl;
    if (cudaMalloc(&st->fbuf, fl * sizeof(float)) != cudaSuccess || cudaMalloc(&st->xbuf, st->xbytes) != cudaSuccess ||
        cudaMallocHost(&st->host_tok, sizeof(int32_t)) != cudaSuccess ||
        cudaMallocHost(&st->host_x, sizeof(float) * c.n_embd) != cudaSuccess) {
        cudaGetLastError();
        bh_stack_free(st);
        return BH_ENOMEM;
    }
    cudaMemsetAsync(st->fbuf, 0, fl * sizeof(float), st->stream);
    cudaMemsetAsync(st->xbuf, 0, st->xbytes, st->stream);
    st->peer_x[rank] = st->xbuf;
    float* F = st->fbuf;
    st->attn_norm = F + o_an; st->ffn_norm = F + o_fn; st->q_norm = F + o_qn; st->k_norm = F + o_kn;
    st->out_norm = F + o_on; st->kc = F + o_kc; st->vc = F + o_vc; st->x_in = F + o_x;
    st->h = reinterpret_cast<float*>(st->xbuf + st->x_h);
    st->attn = reinterpret_cast<float*>(st->xbuf + st->x_attn);
    st->gu = reinterpret_cast<float*>(st->xbuf + st->x_gu);
    st->qkv = F + o_qkv; st->logits = F + o_lg; st->cand_val = F + o_cv;
    st->cand_idx = reinterpret_cast<int32_t*>(F + o_ci);
    st->tok = reinterpret_cast<int32_t*>(F + o_tk);
    st->pos = reinterpret_cast<int*>(F + o_ps);
    st->rope = reinterpret_cast<float2*>(F + o_rf);
    st->cap_h_attn = F + o_ch;
    st->cap_gate_up = F + o_cg;
    {
        // The rotation table, computed the way the reference's CPU backend
        // fills its rope cache (ggml-cpu/ops.cpp ggml_rope_cache_init with
        // freq_scale 1, ext_factor 0, attn_factor 1): theta_scale =
        // powf(base, -2.0f / n_dims); per position theta starts at (float)pos
        // and is multiplied by theta_scale after every pair, in binary32;
        // (cosf(theta), sinf(theta)) with the host C library, as the
        // reference evaluates them.
        const int half = c.head_dim / 2;
        std::vector<float2> rt((size_t)c.n_ctx * half);
        const float theta_scale = powf(c.rope_theta, -2.0f / (float)c.head_dim);
        for (int ps = 0; ps < c.n_ctx; ++ps) {
            volatile float theta = (float)ps;
            for (int i = 0; i < half; ++i) {
                const float th = theta;
                rt[(size_t)ps * half + i] = make_float2(cosf(th), sinf(th));
                theta = th * theta_scale;
            }
        }
        if (cudaMemcpyAsync(st->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, st->stream) !=
                cudaSuccess ||
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
        int64_t r, k, row0;
        mat_dims(st, i < c.n_layer * BH_W_PER_LAYER ? which : -1, &r, &k, &row0);
        const int64_t rows_per_chunk = (int64_t)(chunk_floats / (size_t)k);
        const uint64_t ts = tensor_seed(seed, layer, which);
        // (the values of model rows row0 .. row0 + r - 1: on a row split each
        // rank holds exactly the bytes one GPU holds for those rows)
        for (int64_t r0 = 0; r0 < r && rc == BH_OK; r0 += rows_per_chunk) {
            const int64_t nr = r - r0 < rows_per_chunk ? r - r0 : rows_per_chunk;
            rc = bh::fill_normal(tmp, nr * k, (row0 + r0) * k, ts, 0.0, 0.02, st->stream);
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
    if (st->ctx) cudaSetDevice(st->ctx->device);
    if (st->stream) cudaStreamSynchronize(st->stream);
    if (st->exec) cudaGraphExecDestroy(st->exec);
    if (st->graph) cudaGraphDestroy(st->graph);
    for (int q = 0; q < st->tp_world; ++q)
        if (q != st->tp_rank && st->peer_x[q]) cudaIpcCloseMemHandle(st->peer_x[q]);
    if (st->wbuf) cudaFree(st->wbuf);
    if (st->fbuf) cudaFree(st->fbuf);
    if (st->xbuf) cudaFree(st->xbuf);
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
    const int64_t kvd = (int64_t)c.n_head_kv * c.head_dim;         // the model's KV width
    const int64_t kvd_l = (int64_t)st->n_head_kv_l * c.head_dim;   // this rank's KV heads
    if (cudaSetDevice(st->ctx->device) != cudaSuccess) return BH_ENODEV;
    // on a row split: the model's rows generated whole, this rank's KV heads
    // copied out (the values one GPU holds for them)
    float* tmp = nullptr;
    if (st->tp_world > 1 && n_pos > 0 && cudaMalloc(&tmp, sizeof(float) * (size_t)n_pos * kvd) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    int rc = BH_OK;
    for (int l = 0; l < c.n_layer && rc == BH_OK; ++l) {
        for (int v = 0; v < 2 && rc == BH_OK; ++v) {
            float* dst = (v ? st->vc : st->kc) + (size_t)l * c.n_ctx * kvd_l;
            const uint64_t ts = tensor_seed(seed, l, 100 + v);
            if (!tmp) {
                rc = bh::fill_normal(dst, n_pos * kvd, 0, ts, 0.0, 1.0, st->stream);
                continue;
            }
            rc = bh::fill_normal(tmp, n_pos * kvd, 0, ts, 0.0, 1.0, st->stream);
            if (rc == BH_OK &&
                cudaMemcpy2DAsync(dst, sizeof(float) * kvd_l, tmp + (size_t)st->kh0 * c.head_dim, sizeof(float) * kvd,
                                  sizeof(float) * kvd_l, (size_t)n_pos, cudaMemcpyDeviceToDevice, st->stream) != cudaSuccess)
                rc = BH_EIO;
        }
    }
    if (cudaStreamSynchronize(st->stream) != cudaSuccess) rc = BH_EIO;
    if (tmp) cudaFree(tmp);
    return rc;
}

int bh_stack_tp_handle(bh_stack* st, void* handle_out) {
    if (!st || !handle_out) return BH_EINVAL;
    if (cudaSetDevice(st->ctx->device) != cudaSuccess) return BH_ENODEV;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, st->xbuf) != cudaSuccess) {
        cudaGetLastError();
        return BH_EIO;
    }
    static_assert(sizeof(h) == 64, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    return BH_OK;
}

int bh_stack_tp_connect(bh_stack* st, const void* handles) {
    if (!st || !handles || st->tp_connected) return BH_EINVAL;
    if (cudaSetDevice(st->ctx->device) != cudaSuccess) return BH_ENODEV;
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int q = 0; q < st->tp_world; ++q) {
        if (q == st->tp_rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + 64 * (size_t)q, sizeof(h));
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            for (int r = 0; r < q; ++r)
                if (r != st->tp_rank && st->peer_x[r]) {
                    cudaIpcCloseMemHandle(st->peer_x[r]);
                    st->peer_x[r] = nullptr;
                }
            return BH_EIO;
        }
        st->peer_x[q] = static_cast<uint8_t*>(ptr);
    }
    st->tp_connected = true;
    return BH_OK;
}

int bh_stack_tp_info(bh_stack* st, int* rank, int* world, int64_t* row_ranges) {
    if (!st) return BH_EINVAL;
    if (rank) *rank = st->tp_rank;
    if (world) *world = st->tp_world;
    if (row_ranges) {
        // query heads, KV heads, O / down rows, gate / up rows, LM head rows: (first, count)
        const int64_t v[10] = {st->qh0, st->n_head_l, st->kh0, st->n_head_kv_l, st->e0,
                               st->n_embd_l, st->f0, st->n_ff_l, st->v0, st->n_vocab_l};
        std::memcpy(row_ranges, v, sizeof(v));
    }
    return BH_OK;
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
    if (st->tp_world > 1) return BH_EINVAL;  // one GPU's step only (a row split's launches wait on each other)
    const bh_stack_config& c = st->cfg;
    const int64_t qd = (int64_t)c.n_head * c.head_dim, kvd = (int64_t)c.n_head_kv * c.head_dim;
    int64_t rows = 0, k = 0, xin = 0;
    switch (op) {
        case BH_OP_QKV: rows = qd + 2 * kvd; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
        case BH_OP_O: rows = c.n_embd; k = qd; xin = qd * 4 + (int64_t)c.n_embd * 4; break;
        case BH_OP_GATE_UP: rows = 2 * (int64_t)c.n_ff; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
        case BH_OP_DOWN: rows = c.n_embd; k = c.n_ff; xin = (int64_t)c.n_ff * 4 + (int64_t)c.n_embd * 4; break;
        case BH_OP_ATTN: break;
        default: rows = c.n_vocab; k = c.n_embd; xin = (int64_t)c.n_embd * 8; break;
    }
    if (bytes_per_launch)
        *bytes_per_launch = op == BH_OP_ATTN
                                // q, k, v in; K/V of positions 0..pos (fp32) read; the output written
                                ? (qd + 2 * kvd) * 4 + 2 * (int64_t)c.n_ctx * kvd * 4 + qd * 4
                                : rows * (k / bh::QK) * bh::Q4K_BYTES + xin +
                                      (op == BH_OP_GATE_UP ? (int64_t)c.n_ff : rows) * 4;
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
        mat_dims(st, which, &r, &k);
        *ptr = const_cast<uint8_t*>(st->wq[(size_t)layer * BH_W_PER_LAYER + which]);
    } else if (which == BH_W_OUTPUT) {
        mat_dims(st, -1, &r, &k);
        *ptr = const_cast<uint8_t*>(st->wq[(size_t)c.n_layer * BH_W_PER_LAYER]);
    } else {
        const bool per_layer = which == BH_T_ATTN_NORM || which == BH_T_FFN_NORM || which == BH_T_Q_NORM ||
                               which == BH_T_K_NORM || which == BH_T_K_CACHE || which == BH_T_V_CACHE;
        if (per_layer && (layer < 0 || layer >= c.n_layer)) return BH_EINVAL;
        const int64_t kvd = (int64_t)st->n_head_kv_l * c.head_dim;
        switch (which) {
            case BH_T_ATTN_NORM: *ptr = st->attn_norm + (size_t)layer * c.n_embd; r = 1; k = c.n_embd; break;
            case BH_T_FFN_NORM: *ptr = st->ffn_norm + (size_t)layer * c.n_embd; r = 1; k = c.n_embd; break;
            case BH_T_Q_NORM: *ptr = st->q_norm + (size_t)layer * c.head_dim; r = 1; k = c.head_dim; break;
            case BH_T_K_NORM: *ptr = st->k_norm + (size_t)layer * c.head_dim; r = 1; k = c.head_dim; break;
            case BH_T_OUT_NORM: *ptr = st->out_norm; r = 1; k = c.n_embd; break;
            case BH_T_K_CACHE: *ptr = st->kc + (size_t)layer * c.n_ctx * kvd; r = c.n_ctx; k = kvd; break;
            case BH_T_V_CACHE: *ptr = st->vc + (size_t)layer * c.n_ctx * kvd; r = c.n_ctx; k = kvd; break;
            case BH_T_LOGITS: *ptr = st->logits; r = 1; k = st->n_vocab_l; break;
            case BH_T_HIDDEN: *ptr = st->h; r = 1; k = c.n_embd * (st->tp_world > 1 ? 2 : 1); break;
            case BH_T_QKV: *ptr = st->qkv; r = 1; k = (int64_t)(st->n_head_l + 2 * st->n_head_kv_l) * c.head_dim; break;
            case BH_T_ATTN: *ptr = st->attn; r = 1; k = (int64_t)c.n_head * c.head_dim * (st->tp_world > 1 ? 2 : 1); break;
            case BH_T_H_ATTN: *ptr = st->cap_h_attn; r = 1; k = c.n_embd; break;
            case BH_T_GATE_UP: *ptr = st->cap_gate_up; r = 1; k = 2 * (int64_t)c.n_ff; break;
            case BH_T_FFN_ACT: *ptr = st->gu; r = 1; k = (int64_t)c.n_ff * (st->tp_world > 1 ? 2 : 1); break;
            default: return BH_EINVAL;
        }
    }
    if (rows) *rows = r;
    if (cols) *cols = k;
    return BH_OK;
}

}  // extern "C"
