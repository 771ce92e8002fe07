// q4k_moe.cu — the routed-expert FFN on sm_100a: top-k routing, the grouped
// Q4_K x Q8_K matvecs over the selected experts, SwiGLU and the weighted sum.
//
// The reference's stock block (desktop/engine/src/forward.cpp:1001-1118):
//   probs = soft_max(logits); selected = top_k(probs, k); w = probs[selected],
//   renormalised; up/gate = mul_mat_id(W_up/W_gate, cur); par = silu(gate)*up;
//   down = mul_mat_id(W_down, par); out = sum over the k slots of w * down.
// BURN_MOE (burn_moe_op.cpp:202-372) computes the same block from given
// `selected` / `weights`; both routing sources are supported here.
//
// One cooperative launch per batch of B <= 8 tokens, every CTA resident:
//  1. every CTA routes the batch itself (identical arithmetic, so identical
//     tables) and at once starts streaming both its gate|up rows and its
//     down rows of the U distinct selected experts through its warps' rings
//     (tiles of 8 rows never straddling an expert), so the whole layer's
//     weights are in flight from the start;
//  2. the input columns are RMSNorm'd (when a norm weight is given) and
//     quantized to Q8_K; each gate|up tile computes only the token columns
//     routed to its expert and writes gate | up of those (token, slot) pairs;
//  3. grid barrier; the pairs a CTA's down rows serve are quantized from
//     silu(gate) * up and the down tiles computed from the already-streamed
//     rows; grid barrier;
//  4. out = sum over slots, in order, of (double)(w_s * down_s), rounded
//     once, stored or added to out (the residual stream).
// Each expert's weights are streamed once per batch however many tokens
// chose it. Barrier waits are bounded: on expiry the kernel records a
// timeout in the status word, drains its copies and returns.
#include <cfloat>

#include "bh_common.cuh"
#include "bh_kernels.cuh"
#include "bh_math.cuh"
#include "q4k_core.cuh"
#include "q8k_device.cuh"

namespace bh {

namespace {

// Timeline probe: with BH_TRACE defined, lane 0 of every warp records the
// global timer (ns) at a few points of the kernel into p.trace.
#ifdef BH_TRACE
#define MOE_TRACE_AT(k)                                                                                 \
    do {                                                                                                \
        if (p.trace && (threadIdx.x & 31) == 0) {                                                        \
            uint64_t t_;                                                                                \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            p.trace[((int64_t)blockIdx.x * MV_WARPS + (threadIdx.x >> 5)) * 8 + (k)] = (int64_t)t_;     \
        }                                                                                               \
    } while (0)
// sub-steps of the router, in a second region of the buffer
#define MOE_TRACE_R(k)                                                                                  \
    do {                                                                                                \
        if (p.trace && (threadIdx.x & 31) == 0) {                                                        \
            uint64_t t_;                                                                                \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            p.trace[(4096 + (int64_t)blockIdx.x * MV_WARPS + (threadIdx.x >> 5)) * 8 + (k)] = (int64_t)t_; \
        }                                                                                               \
    } while (0)
#else
#define MOE_TRACE_AT(k) \
    do {                \
    } while (0)
#define MOE_TRACE_R(k) \
    do {               \
    } while (0)
#endif

constexpr int MOE_R = 8;   // rows per tile (TPR = 4)
constexpr int MOE_TPR = 4;

// Routing of one batch, built the same way by every CTA.
struct MoeTable {
    int n_unique;
    int bad;                          // a given expert id out of range, or repeated within a token
    int32_t ids[MOE_MAX_TOK][MOE_MAX_K];
    float w[MOE_MAX_TOK][MOE_MAX_K];
    int16_t expert[MOE_MAX_PAIRS];    // distinct selected experts, ascending
    int8_t cnt[MOE_MAX_PAIRS];        // token columns of each
    int8_t col_tok[MOE_MAX_PAIRS][MOE_MAX_TOK];
    int8_t col_slot[MOE_MAX_PAIRS][MOE_MAX_TOK];
    uint32_t bits[MOE_MAX_EXPERT / 32];
    int base[MOE_MAX_EXPERT / 32];
};

// Shared scratch of the router: probabilities of the batch.
struct __align__(16) RouteScratch {
    float p[MOE_MAX_TOK][MOE_MAX_EXPERT];
    float grp[MOE_MAX_TOK][MOE_MAX_EXPERT / 8];
};

// soft_max -> top_k -> get_rows -> renormalise, for all B tokens of the batch
// (ggml-cpu/ops.cpp:5365-5382 with vec.cpp:547-567; ops.cpp:8157-8194;
// forward.cpp:1032-1046), then the per-expert column lists. All threads of
// the CTA take part; ends with the table complete and a __syncthreads.
// Equal probabilities are ranked lower index first (the reference's
// std::partial_sort leaves their order unspecified). Inputs may have been
// written by an earlier kernel, so they are read around L1.
__device__ __forceinline__ void moe_route(const MoeParams& p, const float* logits, MoeTable& tb,
                                          RouteScratch& rs) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.n_expert, k = p.k, B = p.B;
    if (tid == 0) { tb.bad = 0; tb.n_unique = 0; }
    if (tid < MOE_MAX_EXPERT / 32) tb.bits[tid] = 0;
    if (tid < MOE_MAX_PAIRS) tb.ids[tid / MOE_MAX_K][tid % MOE_MAX_K] = -1;  // a slot left unset is caught below
    __syncthreads();
    if (logits) {
        for (int i = tid; i < B * E; i += MV_THREADS) rs.p[i / E][i % E] = __ldcg(logits + i);
        __syncthreads();
        MOE_TRACE_R(0);
        if (warp < B) {
            float* pr = rs.p[warp];
            float mx = -INFINITY;
            for (int i = lane; i < E; i += 32) mx = fmaxf(mx, pr[i]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            for (int i = lane; i < E; i += 32) pr[i] = exp_ggml(__fsub_rn(pr[i], mx));
            __syncwarp();
            // per-8 fp32 partial sums ((p4+p0)+(p6+p2)) + ((p5+p1)+(p7+p3)), summed in double
            const int ng = E / 8;
            for (int g = lane; g < ng; g += 32) {
                const float* v = pr + 8 * g;
                rs.grp[warp][g] = __fadd_rn(__fadd_rn(__fadd_rn(v[4], v[0]), __fadd_rn(v[6], v[2])),
                                            __fadd_rn(__fadd_rn(v[5], v[1]), __fadd_rn(v[7], v[3])));
            }
            __syncwarp();
            float inv = 0.f;
            if (lane == 0) {
                double sum = 0.0;
                for (int g = 0; g < ng; ++g) sum = __dadd_rn(sum, (double)rs.grp[warp][g]);
                for (int i = 8 * ng; i < E; ++i) sum = __dadd_rn(sum, (double)pr[i]);
                inv = __double2float_rn(__ddiv_rn(1.0, sum));
            }
            inv = __shfl_sync(0xffffffffu, inv, 0);
            for (int i = lane; i < E; i += 32) pr[i] = __fmul_rn(pr[i], inv);
        }
        __syncthreads();
        MOE_TRACE_R(1);
        // top-k of every token: warp b picks its token's k largest
        // probabilities one at a time by a warp-wide argmax (value
        // descending, lower index first on ties) and removes the winner
        if (warp < B) {
            constexpr int PER = MOE_MAX_EXPERT / 32;  // values per lane: index lane + 32 c
            const float* pr = rs.p[warp];
            float pv[PER];
#pragma unroll
            for (int c = 0; c < PER; ++c) pv[c] = lane + 32 * c < E ? pr[lane + 32 * c] : -1.f;  // p >= 0
            for (int s = 0; s < k; ++s) {
                // key = float bits + 1 (order-preserving for p >= 0), 0 once taken
                uint32_t bkey = 0u;
                int bi = 0x7fffffff;
#pragma unroll
                for (int c = 0; c < PER; ++c) {
                    const uint32_t key = pv[c] >= 0.f ? __float_as_uint(pv[c]) + 1u : 0u;
                    if (key > bkey) { bkey = key; bi = lane + 32 * c; }  // increasing index: ties keep the lower
                }
                const uint32_t mkey = __reduce_max_sync(0xffffffffu, bkey);
                bi = (int)__reduce_min_sync(0xffffffffu, bkey == mkey ? (uint32_t)bi : 0xffffffffu);
#pragma unroll
                for (int c = 0; c < PER; ++c)
                    if (lane + 32 * c == bi) pv[c] = -1.f;
                if (lane == 0) tb.ids[warp][(k > 1 && s < 2) ? 1 - s : s] = bi;  // top_k swaps slots 0 and 1
            }
        }
        MOE_TRACE_R(5);
        __syncthreads();
        MOE_TRACE_R(2);
        if (tid < B) {
            float ws[MOE_MAX_K];
            double sum = 0.0;
            for (int s = 0; s < k; ++s) {
                ws[s] = rs.p[tid][tb.ids[tid][s]];
                sum = __dadd_rn(sum, (double)ws[s]);
            }
            const float sf = __double2float_rn(sum);
            for (int s = 0; s < k; ++s) tb.w[tid][s] = p.norm_topk ? __fdiv_rn(ws[s], sf) : ws[s];
        }
    } else {
        for (int i = tid; i < B * k; i += MV_THREADS) {
            tb.ids[i / k][i % k] = __ldcg(p.ids_in + i);
            tb.w[i / k][i % k] = __ldcg(p.w_in + i);
        }
    }
    __syncthreads();
    MOE_TRACE_R(3);
    // distinct experts, ascending: a bitmap, then an exclusive scan of its words
    if (tid < B * k) {
        const int e = tb.ids[tid / k][tid % k];
        if (e < 0 || e >= E) tb.bad = 1;
        else if (e >= p.e_lo && e < p.e_hi) atomicOr(&tb.bits[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = MOE_MAX_EXPERT / 32;
        const uint32_t word = lane < nw ? tb.bits[lane] : 0u;
        const int c = __popc(word);
        int incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += o;
        }
        const int base = incl - c;
        if (lane < nw) {
            tb.base[lane] = base;
            uint32_t wv = word;
            for (int j = 0; wv; ++j) {
                const int bit = __ffs(wv) - 1;
                wv &= wv - 1;
                tb.expert[base + j] = (int16_t)(lane * 32 + bit);
            }
        }
        if (lane == 31) tb.n_unique = incl;
    }
    __syncthreads();
    MOE_TRACE_R(4);
    // column j of pair (t, s) = number of earlier pairs (row-major) on the same expert
    if (tid < B * k) {
        const int t = tid / k, s = tid - t * k;
        const int e = tb.ids[t][s];
        if (e >= 0 && e < E) {
            const int u = tb.base[e >> 5] + __popc(tb.bits[e >> 5] & ((1u << (e & 31)) - 1u));
            int j = 0, n = 0;
            for (int q = 0; q < B * k; ++q) {
                const int same = tb.ids[q / k][q % k] == e;
                j += same & (q < tid);
                n += same;
            }
            if (n > B) tb.bad = 1;  // an expert repeated within one token's selection
            else if (e >= p.e_lo && e < p.e_hi) {
                tb.col_tok[u][j] = (int8_t)t;
                tb.col_slot[u][j] = (int8_t)s;
                if (j == 0) tb.cnt[u] = (int8_t)n;
            }
        }
    }
    __syncthreads();
}

// The token values (and norm weights) of this warp's block, loaded before the
// routing when every warp has at most one block (one token): their L2 round
// trip then overlaps the router instead of following it.
struct TokPre {
    float v[8], g[8];
    bool have;
};

__device__ __forceinline__ void preload_tokens(const MoeParams& p, const float* gamma, TokPre& t) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.n_embd / QK, nblk = p.B * nb;
    t.have = nblk <= MV_WARPS;
#pragma unroll
    for (int j = 0; j < 8; ++j) { t.v[j] = 0.f; t.g[j] = 0.f; }
    if (!t.have || warp >= nblk) return;
    const int b = warp / nb, i = warp - b * nb;
    const int e0 = i * QK + 8 * lane;
    const float4* x = reinterpret_cast<const float4*>(p.h + (int64_t)b * p.n_embd + e0);
    const float4 a0 = __ldcg(x), a1 = __ldcg(x + 1);
    t.v[0] = a0.x; t.v[1] = a0.y; t.v[2] = a0.z; t.v[3] = a0.w;
    t.v[4] = a1.x; t.v[5] = a1.y; t.v[6] = a1.z; t.v[7] = a1.w;
    if (gamma) {
        const uint64_t keep = policy_evict_last();
        const float4 g0 = ldg_f4_keep(gamma + e0, keep), g1 = ldg_f4_keep(gamma + e0 + 4, keep);
        t.g[0] = g0.x; t.g[1] = g0.y; t.g[2] = g0.z; t.g[3] = g0.w;
        t.g[4] = g1.x; t.g[5] = g1.y; t.g[6] = g1.z; t.g[7] = g1.w;
    }
}

// Gate|up prologue: the B input columns, RMSNorm'd when a weight is given
// (ggml rms_norm: fp32 squares summed in double, mean = (float)(sum / n),
// scale = 1 / sqrt(mean + eps), y = (x * scale) * gamma), quantized to Q8_K.
template <int FOLD>
__device__ void stage_tokens(const MoeParams& p, const float* gamma, uint8_t* act, float* s_scale, const TokPre& pre) {
    __shared__ double s_bss[MOE_MAX_TOK * MOE_MAX_EMBD_BLOCKS];  // per-block sums of squares
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.n_embd, nb = K / QK;
    const int nblk = p.B * nb;
    // Every warp takes blocks warp, warp + MV_WARPS, ... and issues all the
    // loads of a round (h, gamma) before using any: the activations were just
    // written by another kernel, so each round trip to the L2 is paid once
    // per round. With RMSNorm the per-block sums of squares (lane sums and a
    // butterfly, in double) are combined per token in block order; when one
    // round covers every block the values wait in registers for the scale.
    constexpr int UF = 4;
    const bool one_round = nblk <= MV_WARPS * UF;
    const int rounds = (nblk + MV_WARPS * UF - 1) / (MV_WARPS * UF);  // the same in every warp
    const uint64_t keep = policy_evict_last();
    auto scales = [&]() {
        __syncthreads();
        if (threadIdx.x < p.B) {
            double ss = 0.0;
            for (int i = 0; i < nb; ++i) ss = __dadd_rn(ss, s_bss[threadIdx.x * nb + i]);
            const float mean = __double2float_rn(div_by_count(ss, K));
            s_scale[threadIdx.x] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        }
        __syncthreads();
    };
    auto put = [&](int blk, const float (&x)[8]) {
        const Q8Block qb = q8k_quantize_warp(x, lane);
        uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
        stage_codes<FOLD>(dst, qb.q, lane);
        stage_scalars(dst, qb.d, qb.bsum16, lane);
    };
    for (int rd = 0; rd < rounds; ++rd) {
        const int blk0 = warp + rd * MV_WARPS * UF;
        float v[UF][8], g[UF][8];
#pragma unroll
        for (int u = 0; u < UF; ++u) {
            const int blk = blk0 + u * MV_WARPS;
            const int b = blk / nb, i = blk - b * nb;
            const int e0 = i * QK + 8 * lane;
            float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, g0 = a0, g1 = a0;
            if (pre.have) {
                // (one block per warp, loaded before the routing)
                if (u == 0) {
                    a0 = make_float4(pre.v[0], pre.v[1], pre.v[2], pre.v[3]);
                    a1 = make_float4(pre.v[4], pre.v[5], pre.v[6], pre.v[7]);
                    g0 = make_float4(pre.g[0], pre.g[1], pre.g[2], pre.g[3]);
                    g1 = make_float4(pre.g[4], pre.g[5], pre.g[6], pre.g[7]);
                }
            } else if (blk < nblk) {
                const float4* x = reinterpret_cast<const float4*>(p.h + (int64_t)b * K + e0);
                a0 = __ldcg(x);
                a1 = __ldcg(x + 1);
                if (gamma) {
                    g0 = ldg_f4_keep(gamma + e0, keep);
                    g1 = ldg_f4_keep(gamma + e0 + 4, keep);
                }
            }
            v[u][0] = a0.x; v[u][1] = a0.y; v[u][2] = a0.z; v[u][3] = a0.w;
            v[u][4] = a1.x; v[u][5] = a1.y; v[u][6] = a1.z; v[u][7] = a1.w;
            g[u][0] = g0.x; g[u][1] = g0.y; g[u][2] = g0.z; g[u][3] = g0.w;
            g[u][4] = g1.x; g[u][5] = g1.y; g[u][6] = g1.z; g[u][7] = g1.w;
        }
        if (!gamma) {
#pragma unroll
            for (int u = 0; u < UF; ++u)
                if (blk0 + u * MV_WARPS < nblk) put(blk0 + u * MV_WARPS, v[u]);
            continue;
        }
#pragma unroll
        for (int u = 0; u < UF; ++u) {
            double ss = 0.0;
#pragma unroll
            for (int t = 0; t < 8; ++t) ss = __dadd_rn(ss, (double)__fmul_rn(v[u][t], v[u][t]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if (lane == 0 && blk0 + u * MV_WARPS < nblk) s_bss[blk0 + u * MV_WARPS] = ss;
        }
        if (one_round) {
            scales();
#pragma unroll
            for (int u = 0; u < UF; ++u) {
                const int blk = blk0 + u * MV_WARPS;
                if (blk >= nblk) continue;  // warp-uniform
                const float sc = s_scale[blk / nb];
                float x[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) x[t] = __fmul_rn(__fmul_rn(v[u][t], sc), g[u][t]);
                put(blk, x);
            }
        }
    }
    if (!gamma || one_round) return;
    // several rounds (many tokens or a wide embedding): the scales from the
    // block sums, then the blocks loaded again and quantized
    scales();
    for (int blk = warp; blk < nblk; blk += MV_WARPS) {
        const int b = blk / nb, i = blk - b * nb;
        const int e0 = i * QK + 8 * lane;
        const float4* x = reinterpret_cast<const float4*>(p.h + (int64_t)b * K + e0);
        const float4 a0 = __ldcg(x), a1 = __ldcg(x + 1);
        const float4 g0 = ldg_f4_keep(gamma + e0, keep), g1 = ldg_f4_keep(gamma + e0 + 4, keep);
        const float hv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float sc = s_scale[b];
        float xv[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) xv[t] = __fmul_rn(__fmul_rn(hv[t], sc), gv[t]);
        put(blk, xv);
    }
}

// Down prologue: silu(gate) * up of the pairs of experts u_lo..u_hi (written
// by other CTAs before the grid barrier, so read around L1), pair q of this
// CTA staged at act + q * nb blocks.
template <int FOLD>
__device__ void stage_pairs(const MoeParams& p, const MoeTable& tb, int u_lo, int u_hi, uint8_t* act,
                            int* s_qbase) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.n_ff / QK;
    if (threadIdx.x == 0) {
        int q = 0;
        for (int u = u_lo; u <= u_hi; ++u) { s_qbase[u - u_lo] = q; q += tb.cnt[u]; }
        s_qbase[u_hi - u_lo + 1] = q;
    }
    __syncthreads();
    const int npairs = s_qbase[u_hi - u_lo + 1];
    const int nblk = npairs * nb;
    // UF blocks per warp per round, all their loads issued before any use
    constexpr int UF = 4;
    for (int blk0 = warp; blk0 < nblk; blk0 += MV_WARPS * UF) {
        float4 ld[UF][4];
#pragma unroll
        for (int r = 0; r < UF; ++r) {
            const int blk = blk0 + r * MV_WARPS;
            ld[r][0] = ld[r][1] = ld[r][2] = ld[r][3] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (blk < nblk) {
                const int q = blk / nb, i = blk - q * nb;
                int u = u_lo;
                while (u < u_hi && s_qbase[u + 1 - u_lo] <= q) ++u;
                const int j = q - s_qbase[u - u_lo];
                const int pair = tb.col_tok[u][j] * p.k + tb.col_slot[u][j];
                const int e0 = i * QK + 8 * lane;
                const float4* g = reinterpret_cast<const float4*>(p.gu + (int64_t)pair * 2 * p.n_ff + e0);
                const float4* up = reinterpret_cast<const float4*>(p.gu + (int64_t)pair * 2 * p.n_ff + p.n_ff + e0);
                ld[r][0] = __ldcg(g);
                ld[r][1] = __ldcg(g + 1);
                ld[r][2] = __ldcg(up);
                ld[r][3] = __ldcg(up + 1);
            }
        }
#pragma unroll
        for (int r = 0; r < UF; ++r) {
            const int blk = blk0 + r * MV_WARPS;
            if (blk >= nblk) break;  // warp-uniform
            const float gv[8] = {ld[r][0].x, ld[r][0].y, ld[r][0].z, ld[r][0].w,
                                 ld[r][1].x, ld[r][1].y, ld[r][1].z, ld[r][1].w};
            const float uv[8] = {ld[r][2].x, ld[r][2].y, ld[r][2].z, ld[r][2].w,
                                 ld[r][3].x, ld[r][3].y, ld[r][3].z, ld[r][3].w};
            float v[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(silu_ggml(gv[t]), uv[t]);
            const Q8Block qb = q8k_quantize_warp(v, lane);
            uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
            stage_codes<FOLD>(dst, qb.q, lane);
            stage_scalars(dst, qb.d, qb.bsum16, lane);
        }
    }
}

// Grid-wide barrier of a cooperative launch (every CTA resident). Writes of
// the CTA before the barrier are visible to every CTA after it. Self-resetting:
// the last arrival zeroes the count and advances the generation the others
// wait on, in one atomic on the same word. The wait is bounded; false after a
// timeout (status recorded).
__device__ bool grid_barrier(unsigned int* gbar, int* status, long long wait_cycles) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        // one word: arrivals in the low 16 bits, the generation above them
        __threadfence();
        const unsigned int old = atomicAdd(gbar, 1u);
        const unsigned int gen = old >> 16;
        int ok = 1;
        if ((old & 0xffffu) == gridDim.x - 1) {
            atomicAdd(gbar, (1u << 16) - gridDim.x);  // count back to zero, next generation
            __threadfence();
        } else {
            const long long t0 = clock64();
            for (;;) {
                unsigned int g;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(gbar) : "memory");
                if ((g >> 16) != gen) break;
                if (clock64() - t0 > wait_cycles) {
                    ok = 0;
                    set_status(status, ST_TIMEOUT);
                    break;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// Tiles of the CTA in one phase: a contiguous range of the phase's 8-row
// tiles over the U selected experts.
struct PhaseRange {
    int t_begin, t_end, te;  // tile range, tiles per expert
    __device__ int mine(int warp) const {
        const int n = t_end - t_begin;
        return warp < n ? (n - 1 - warp) / MV_WARPS + 1 : 0;
    }
};

// Work the blocks of one ring slot for this thread's row: TPR threads per
// row, NB-bounded token columns.
template <int FOLD, int NB>
__device__ __forceinline__ void tile_fold(const uint8_t* rowp, int kl, const uint8_t* act_base, int nb,
                                          const int (&colbase)[NB], int cols, int t, float (&acc)[NB][8 / MOE_TPR],
                                          float (&accm)[NB], int sbc) {
#pragma unroll 2
    for (int kb = 0; kb < kl; ++kb) {
        const RowBlk<MOE_TPR> r = decode_row<FOLD, MOE_TPR>(rowp + kb * Q4K_BYTES, t);
#pragma unroll
        for (int c = 0; c < NB; ++c)
            if (c < cols)
                fold_block<FOLD, false, MOE_TPR>(r, act_base + (colbase[c] * nb + sbc + kb) * ACT_BLOCK_BYTES, t,
                                                 nullptr, acc[c], accm[c]);
    }
}

// The fused routed-expert FFN of one batch (see the file comment).
template <int FOLD, int NB>
__global__ void __launch_bounds__(MV_THREADS, 1) q4k_moe_kernel(const __grid_constant__ MoeParams p) {
    constexpr int R = MOE_R, TPR = MOE_TPR, L = 8 / TPR;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ MoeTable tb;
    __shared__ RouteScratch rs;
    __shared__ float s_scale[MOE_MAX_TOK];
    __shared__ int s_qbase[MOE_MAX_PAIRS + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned FULLM = 0xffffffffu;
    if (threadIdx.x == 0) {
        prefetch_tmap(&p.tmap[0]);
        prefetch_tmap(&p.tmap[1]);
        prefetch_tmap(&p.tmap[2]);
    }
    pdl_wait();  // routing inputs and h may come from the previous kernel
    pdl_trigger();

    uint8_t* act = smem + p.act_off;
    uint8_t* ring = smem + p.ring_off + (size_t)warp * p.stages * p.slot_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off) + warp * p.stages;
    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const uint64_t pol = policy_evict_first();
    const int nb_e = p.n_embd / QK, nb_f = p.n_ff / QK;
    const int nkc_gu = (nb_e + p.kc_gu - 1) / p.kc_gu, nkc_dn = (nb_f + p.kc_dn - 1) / p.kc_dn;
    const int rgrp = lane / TPR;
    const int t = lane % TPR;
    // ring cursors run on across layers: every layer consumes all it issues
    int c_s = 0, i_s = 0;
    uint32_t c_ph = 0;
    bool ok = true;

    for (int l = 0; l < p.n_layer; ++l) {
        MOE_TRACE_AT(0);
        const float* gamma_l = p.gamma ? p.gamma + l * p.gamma_ls : nullptr;
        TokPre pre;
        preload_tokens(p, gamma_l, pre);
        moe_route(p, p.logits ? p.logits + l * p.logits_ls : nullptr, tb, rs);
        MOE_TRACE_AT(1);
        if (tb.bad) {
            if (threadIdx.x == 0) set_status(p.status, ST_BADARG);
            return;  // uniform over the grid: every CTA built the same table
        }
        if (blockIdx.x == 0 && threadIdx.x < p.B * p.k) {
            const int tk = threadIdx.x / p.k, s = threadIdx.x - tk * p.k;
            if (p.ids_out) p.ids_out[l * p.route_ls + threadIdx.x] = tb.ids[tk][s];
            if (p.w_out) p.w_out[l * p.route_ls + threadIdx.x] = tb.w[tk][s];
        }

        if (!p.combine) {
            // rows of pairs on other ranks' experts: -0.0, the identity of the cross-rank sum
            const int np = p.B * p.k * p.n_embd;
            for (int idx = blockIdx.x * MV_THREADS + threadIdx.x; idx < np; idx += gridDim.x * MV_THREADS) {
                const int q = idx / p.n_embd;
                const int e = tb.ids[q / p.k][q % p.k];
                if (e < p.e_lo || e >= p.e_hi) p.dout[idx] = -0.f;
            }
        }
        const int U = tb.n_unique;
        const int ebase = l * (p.e_hi - p.e_lo);  // bank row blocks of this layer
        PhaseRange gu, dn;
        gu.te = 2 * p.n_ff / R;
        dn.te = p.n_embd / R;
        gu.t_begin = (int)((int64_t)U * gu.te * blockIdx.x / gridDim.x);
        gu.t_end = (int)((int64_t)U * gu.te * (blockIdx.x + 1) / gridDim.x);
        dn.t_begin = (int)((int64_t)U * dn.te * blockIdx.x / gridDim.x);
        dn.t_end = (int)((int64_t)U * dn.te * (blockIdx.x + 1) / gridDim.x);
        const int my_gu = gu.mine(warp), my_dn = dn.mine(warp);
        const int total = my_gu * nkc_gu + my_dn * nkc_dn;

        // one issue cursor over the warp's gate|up tiles, then its down tiles
        int i_ph = my_gu > 0 ? 0 : 1, i_j = 0, i_c = 0, issued = 0;
        auto issue_next = [&]() {
            if (lane == 0) {
                int map, x;
                int64_t row;
                uint32_t bytes;
                if (i_ph == 0) {
                    const int tile = gu.t_begin + warp + i_j * MV_WARPS;
                    const int u = tile / gu.te, rt = (tile - u * gu.te) * R;
                    map = rt >= p.n_ff;
                    row = (int64_t)(ebase + tb.expert[u] - p.e_lo) * p.n_ff + (map ? rt - p.n_ff : rt);
                    x = i_c * p.kc_gu * (Q4K_BYTES / 8);
                    bytes = (uint32_t)p.stage_gu;
                } else {
                    const int tile = dn.t_begin + warp + i_j * MV_WARPS;
                    const int u = tile / dn.te, rt = (tile - u * dn.te) * R;
                    map = 2;
                    row = (int64_t)(ebase + tb.expert[u] - p.e_lo) * p.n_embd + rt;
                    x = i_c * p.kc_dn * (Q4K_BYTES / 8);
                    bytes = (uint32_t)p.stage_dn;
                }
                mbar_arrive_expect_tx(&full[i_s], bytes);
                tensor_g2s_2d(ring + (size_t)i_s * p.slot_bytes, &p.tmap[map], x, (int)row, &full[i_s], pol);
            }
            __syncwarp();
            ++issued;
            if (++i_c == (i_ph == 0 ? nkc_gu : nkc_dn)) {
                i_c = 0;
                if (++i_j == my_gu && i_ph == 0) { i_ph = 1; i_j = 0; }
            }
            if (++i_s == p.stages) i_s = 0;
        };
        // two stages per warp now, the rest of the ring once the token
        // activations are staged (their loads then do not queue behind a full
        // ring of weight copies)
        const int ring_fill = min(p.stages, total);
        MOE_TRACE_R(6);
        for (int q = 0; q < min(2, ring_fill); ++q) {
            issue_next();
            if (q == 0) MOE_TRACE_R(7);
        }
        MOE_TRACE_AT(2);

        stage_tokens<FOLD>(p, gamma_l, act, s_scale, pre);
        while (issued < ring_fill) issue_next();
        __syncthreads();
        MOE_TRACE_AT(3);

        int consumed = 0;
        auto wait_slot = [&]() -> bool {
            if (!__all_sync(FULLM, mbar_wait_bounded(&full[c_s], c_ph))) {
                if (lane == 0) set_status(p.status, ST_TIMEOUT);
                return false;
            }
#ifdef BH_TRACE
            if (consumed == 0) MOE_TRACE_AT(4);
#endif
            ++consumed;
            return true;
        };
        auto release_slot = [&]() {
            __syncwarp();
            if (issued < total) {
                fence_proxy_async_smem();
                issue_next();
            }
            if (++c_s == p.stages) { c_s = 0; c_ph ^= 1u; }
        };

        // ---- the two matvec phases share one tile loop (one copy of the
        // code): phase 0 gate | up over the token columns, then a grid
        // barrier and the staging of the down columns, phase 1 down over the
        // (token, slot) pairs
        const int u_lo = dn.t_end > dn.t_begin ? dn.t_begin / dn.te : 0;
        const int u_hi = dn.t_end > dn.t_begin ? (dn.t_end - 1) / dn.te : 0;
        for (int ph = 0; ph < 2; ++ph) {
            if (ph == 1) {
                MOE_TRACE_AT(5);
                ok = grid_barrier(p.gbar, p.status, p.gbar_wait) && ok;
                if (dn.t_end > dn.t_begin && __syncthreads_and(ok)) stage_pairs<FOLD>(p, tb, u_lo, u_hi, act, s_qbase);
                __syncthreads();
                MOE_TRACE_AT(6);
            }
            const PhaseRange& pr = ph == 0 ? gu : dn;
            const int mine = ph == 0 ? my_gu : my_dn;
            const int kc = ph == 0 ? p.kc_gu : p.kc_dn, stride = ph == 0 ? p.stride_gu : p.stride_dn;
            const int nb = ph == 0 ? nb_e : nb_f, nkc = ph == 0 ? nkc_gu : nkc_dn;
            float* const obase = ph == 0 ? p.gu : p.dout;
            const int64_t ostride = ph == 0 ? 2 * (int64_t)p.n_ff : (int64_t)p.n_embd;
            for (int j = 0; j < mine && ok; ++j) {
                const int tile = pr.t_begin + warp + j * MV_WARPS;
                const int u = tile / pr.te, rt = (tile - u * pr.te) * R;
                const int cols = tb.cnt[u];
                int colbase[NB];
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    const int cc = c < cols ? c : 0;
                    colbase[c] = ph == 0 ? tb.col_tok[u][cc] : s_qbase[u - u_lo] + cc;
                }
                float acc[NB][L], accm[NB];
#pragma unroll
                for (int c = 0; c < NB; ++c) {
#pragma unroll
                    for (int e = 0; e < L; ++e) acc[c][e] = 0.f;
                    accm[c] = 0.f;
                }
                for (int ci = 0; ci < nkc; ++ci) {
                    if (!(ok = wait_slot())) break;
                    const int sbc = ci * kc;
                    tile_fold<FOLD, NB>(ring + (size_t)c_s * p.slot_bytes + (size_t)rgrp * stride, min(kc, nb - sbc),
                                        act, nb, colbase, cols, t, acc, accm, sbc);
                    release_slot();
                }
                if (!ok) break;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    if (c < cols) {
                        const float v = row_value<FOLD, TPR>(acc[c], accm[c], rgrp);
                        if (t == 0) {
                            const int pair = tb.col_tok[u][c] * p.k + tb.col_slot[u][c];
                            obase[(int64_t)pair * ostride + rt + rgrp] = v;
                        }
                    }
                }
            }
        }
        if (!ok && lane == 0) {
            // nothing of this warp may still be in flight when the CTA exits
            int s = c_s;
            uint32_t ph = c_ph;
            for (int q = consumed; q < issued; ++q) {
                mbar_wait_bounded(&full[s], ph);
                if (++s == p.stages) { s = 0; ph ^= 1u; }
            }
        }
        MOE_TRACE_AT(7);
        if (!p.combine) return;  // the caller sums dout over the ranks, then combines
        ok = grid_barrier(p.gbar, p.status, p.gbar_wait) && ok;
        if (!__syncthreads_and(ok)) return;

        // ---- combine: ggml_mul (fp32 product) then ggml_sum_rows over the
        // slots (double, in slot order), rounded once; this CTA's slice
        const int n = p.B * p.n_embd;
        const int per = (n + gridDim.x - 1) / gridDim.x;
        const int e_end = min(n, (int)(blockIdx.x + 1) * per);
        for (int idx = blockIdx.x * per + threadIdx.x; idx < e_end; idx += MV_THREADS) {
            const int tk = idx / p.n_embd, i = idx - tk * p.n_embd;
            double a = 0.0;
            for (int s = 0; s < p.k; ++s)
                a = __dadd_rn(a, (double)__fmul_rn(__ldcg(p.dout + ((int64_t)tk * p.k + s) * p.n_embd + i), tb.w[tk][s]));
            const float r = __double2float_rn(a);
            p.out[idx] = p.residual ? __fadd_rn(p.out[idx], r) : r;
        }
        // the next layer's RMSNorm reads every CTA's slice of h
        if (l + 1 < p.n_layer && !grid_barrier(p.gbar, p.status, p.gbar_wait)) return;
    }
}

// Routing alone (one CTA): ids / weights of the batch.
__global__ void __launch_bounds__(MV_THREADS, 1) moe_route_kernel(const __grid_constant__ MoeParams p) {
    __shared__ MoeTable tb;
    __shared__ RouteScratch rs;
    pdl_wait();
    pdl_trigger();
    moe_route(p, p.logits, tb, rs);
    if (tb.bad) {
        if (threadIdx.x == 0) set_status(p.status, ST_BADARG);
        return;
    }
    if (threadIdx.x < p.B * p.k) {
        const int t = threadIdx.x / p.k, s = threadIdx.x - t * p.k;
        p.ids_out[threadIdx.x] = tb.ids[t][s];
        p.w_out[threadIdx.x] = tb.w[t][s];
    }
}

// (dout2, when set: a pair's row is dout + dout2, one of them holding the
// expert output and the other -0.0, which makes the sum that value exactly)
__global__ void __launch_bounds__(256) moe_combine_kernel(const float* __restrict__ dout, const float* __restrict__ dout2,
                                                          const float* __restrict__ w, int B, int k, int n_embd,
                                                          float* out, int residual) {
    pdl_wait();
    pdl_trigger();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * n_embd) return;
    const int t = idx / n_embd, i = idx - t * n_embd;
    // ggml_mul (fp32 product) then ggml_sum_rows over the slots (double, in order)
    double a = 0.0;
    for (int s = 0; s < k; ++s) {
        const int64_t o = ((int64_t)t * k + s) * n_embd + i;
        const float e = dout2 ? __fadd_rn(__ldcg(dout + o), __ldcg(dout2 + o)) : __ldcg(dout + o);
        a = __dadd_rn(a, (double)__fmul_rn(e, __ldcg(w + t * k + s)));
    }
    const float r = __double2float_rn(a);
    out[idx] = residual ? __fadd_rn(out[idx], r) : r;
}

}  // namespace

// Shared-memory plan: the activation region (B token columns of n_embd, or
// up to B*k pairs of n_ff, whichever is larger), then per warp `stages` ring
// slots sized for the larger phase stage, then the mbarriers. kc per phase
// from the copy target (box rows stay within 2048 bytes).
int moe_plan(MoeParams& p, int smem_cap, int stage_target) {
    const int nb_e = p.n_embd / QK, nb_f = p.n_ff / QK;
    p.act_blocks = max(p.B * nb_e, p.B * p.k * nb_f);
    const int act_bytes = p.act_blocks * ACT_BLOCK_BYTES;
    const int ring_off = (act_bytes + 127) / 128 * 128;
    auto stride_for = [](int kc) {
        const int words = kc * (Q4K_BYTES / 4);
        const int padw = ((8 - (words % 32)) % 32 + 32) % 32;  // row stride == 8 words (mod 32 banks)
        return kc * Q4K_BYTES + 4 * padw;
    };
    int kc = stage_target / Q4K_BYTES;
    if (kc < 1) kc = 1;
    if (kc > 13) kc = 13;
    for (; kc >= 1; --kc) {
        const int kg = min(kc, nb_e), kd = min(kc, nb_f);
        const int sg = MOE_R * stride_for(kg), sd = MOE_R * stride_for(kd);
        const int slot = max(sg, sd);
        const int avail = smem_cap - ring_off - 128;
        int stages = avail > 0 ? avail / (MV_WARPS * (slot + 8)) : 0;
        if (stages > 8) stages = 8;
        if (stages < 2) continue;
        p.kc_gu = kg;
        p.stride_gu = stride_for(kg);
        p.stage_gu = sg;
        p.kc_dn = kd;
        p.stride_dn = stride_for(kd);
        p.stage_dn = sd;
        p.slot_bytes = slot;
        p.stages = stages;
        p.act_off = 0;
        p.ring_off = ring_off;
        p.bar_off = ring_off + MV_WARPS * stages * slot;
        p.smem_bytes = p.bar_off + MV_WARPS * stages * 8;
        return BH_OK;
    }
    return BH_EINVAL;
}

template <int FOLD, int NB>
static int launch_moe_t(const MoeParams& p, const LaunchOpts& o) {
    auto kern = q4k_moe_kernel<FOLD, NB>;
    static std::atomic<uint64_t> attr_devices{0};
    if (!attrs_on_device(attr_devices, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
                       cudaSuccess &&
                   cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared) == cudaSuccess;
        }))
        return BH_EIO;
    // every CTA must be resident (grid barriers): clamp to what fits
    int dev = 0, nsm = 0, occ = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, MV_THREADS, (size_t)p.smem_bytes) != cudaSuccess ||
        occ < 1)
        return BH_EIO;
    const int grid = min(o.grid, nsm * occ);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = (size_t)p.smem_bytes;
    cfg.stream = o.stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = o.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? BH_OK : BH_EIO;
}

template <int FOLD>
static int launch_moe_nb(const MoeParams& p, const LaunchOpts& o) {
    // NB bounds the token columns of one expert (at most B)
    if (p.B <= 1) return launch_moe_t<FOLD, 1>(p, o);
    if (p.B <= 2) return launch_moe_t<FOLD, 2>(p, o);
    if (p.B <= 4) return launch_moe_t<FOLD, 4>(p, o);
    return launch_moe_t<FOLD, 8>(p, o);
}

int launch_moe(const MoeParams& pin, int fold, const LaunchOpts& o) {
    if (o.grid < 1 || pin.B < 1 || pin.B > MOE_MAX_TOK || pin.k < 1 || pin.k > MOE_MAX_K ||
        pin.n_expert < pin.k || pin.n_expert > MOE_MAX_EXPERT || pin.n_ff % QK || pin.n_embd % QK || !pin.gbar ||
        !pin.gu || !pin.dout || pin.n_layer < 1 || (pin.n_layer > 1 && (!pin.residual || !pin.combine)) ||
        (pin.combine && !pin.out) || pin.e_lo < 0 || pin.e_hi > pin.n_expert || pin.e_lo >= pin.e_hi ||
        (int64_t)pin.n_layer * pin.n_expert * (pin.n_ff > pin.n_embd ? pin.n_ff : pin.n_embd) >= ((int64_t)1 << 31))
        return BH_EINVAL;
    MoeParams p = pin;
    const int nb_e = p.n_embd / QK, nb_f = p.n_ff / QK;
    const int64_t ne = (int64_t)p.n_layer * (p.e_hi - p.e_lo);
    int rc = encode_q4k_map(&p.tmap[0], p.w[0], ne * p.n_ff, nb_e, p.stride_gu, MOE_R);
    if (rc == BH_OK) rc = encode_q4k_map(&p.tmap[1], p.w[1], ne * p.n_ff, nb_e, p.stride_gu, MOE_R);
    if (rc == BH_OK) rc = encode_q4k_map(&p.tmap[2], p.w[2], ne * p.n_embd, nb_f, p.stride_dn, MOE_R);
    if (rc != BH_OK) return rc;
    if (fold == BH_FOLD_X86) return launch_moe_nb<BH_FOLD_X86>(p, o);
    if (fold == BH_FOLD_GENERIC) return launch_moe_nb<BH_FOLD_GENERIC>(p, o);
    return BH_EINVAL;
}

int launch_moe_combine(const float* dout, const float* w, int B, int k, int n_embd, float* out, bool residual,
                       const LaunchOpts& o, const float* dout2) {
    const int n = B * n_embd;
    if (n < 1 || k < 1 || !dout || !w || !out) return BH_EINVAL;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = o.stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = o.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, moe_combine_kernel, dout, dout2, w, B, k, n_embd, out, residual ? 1 : 0) ==
                   cudaSuccess
               ? BH_OK
               : BH_EIO;
}

int launch_moe_route(const MoeParams& p, const LaunchOpts& o) {
    if (p.B < 1 || p.B > MOE_MAX_TOK || p.k < 1 || p.k > MOE_MAX_K || p.n_expert < p.k ||
        p.n_expert > MOE_MAX_EXPERT || !p.logits || !p.ids_out || !p.w_out)
        return BH_EINVAL;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.stream = o.stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = o.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, moe_route_kernel, p) == cudaSuccess ? BH_OK : BH_EIO;
}

}  // namespace bh
