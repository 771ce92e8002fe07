// q4k_matvec.cu — the sm_100a Q4_K x Q8_K matvec (batch 1..8).
//
// Structure (16 warps per CTA at batch 1-2 and for narrow matrices at batch
// 3-8, else 8; 1 or 2 CTAs per SM, each CTA persistent over a contiguous
// range of rows):
//  - every warp owns tiles of 32/TPR consecutive rows and streams them
//    through its own ring of shared-memory stages: one 2-D tensor copy
//    (cp.async.bulk.tensor, the TMA engine) per stage, issued by lane 0 and
//    counted on the stage's mbarrier, rows padded so reads are bank-conflict
//    free. All warps issue copies in parallel; weights do not depend on the
//    previous kernel, so each warp starts streaming before the programmatic-
//    launch wait.
//  - all warps stage the activations once (Q8_K input, or fp32 input
//    quantized in the prologue, optionally through RMSNorm), then
//    TPR threads work each row; the per-block arithmetic (q4k_core.cuh)
//    reproduces the reference's integer sums and fp32 fold bit for bit.
#include "bh_common.cuh"
#include "bh_kernels.cuh"
#include "bh_math.cuh"
#include "q4k_core.cuh"
#include "q8k_device.cuh"

// Super-blocks of one stage worked per unrolled step of a warp (the integer
// work of consecutive blocks is independent; only the fp32 fold chains them).
#ifndef BH_KB_UNROLL
#define BH_KB_UNROLL 2
#endif
#define BH_STR_(x) #x
#define BH_UNROLL(n) _Pragma(BH_STR_(unroll n))

namespace bh {

// Timeline probe: with BH_TRACE defined, lane 0 of every warp records the
// global timer (ns) at a few points of the kernel into p.trace.
#ifdef BH_TRACE
#define BH_TRACE_AT(k)                                                                                  \
    do {                                                                                                \
        if (p.trace && (threadIdx.x & 31) == 0) {                                                        \
            uint64_t t_;                                                                                \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            p.trace[((int64_t)blockIdx.x * DENSE_MAX_WARPS + (threadIdx.x >> 5)) * 8 + (k)] = (int64_t)t_; \
        }                                                                                               \
    } while (0)
#else
#define BH_TRACE_AT(k) \
    do {               \
    } while (0)
#endif

// Segment holding virtual row `row` (segment boundaries are multiples of 8,
// so an oct never straddles two) and the row's index within it.
__device__ __forceinline__ int seg_of(const MatvecParams& p, int64_t row, int64_t& local) {
    if (row < p.seg_end[0]) { local = row; return 0; }
    if (row < p.seg_end[1]) { local = row - p.seg_end[0]; return 1; }
    local = row - p.seg_end[1];
    return 2;
}

// ---------------------------------------------------------------------------
// prologue: activations -> staged Q8_K blocks in shared memory
// ---------------------------------------------------------------------------
// Blocks per warp per staging round of fp32 sources: with 16 warps one round
// covers the decode step's prologues at batch 1 (RMSNorm K <= 8192, plain
// quantize K <= 12288).
constexpr int STAGE_UF = 2;  // RMSNorm
template <int SRC>
__host__ __device__ constexpr int stage_uf() { return SRC == ACT_F32_RMSNORM ? STAGE_UF : 3; }

// RMSNorm weights of this warp's first-round blocks (they do not depend on the
// previous kernel, so they are loaded before the programmatic wait, ahead of
// the weight copies).
template <int W>
__device__ __forceinline__ void preload_gamma(const MatvecParams& p, float (&gp)[STAGE_UF][8],
                                              int warp, int lane) {
    constexpr int UF = STAGE_UF;
    const uint64_t keep = policy_evict_last();
#pragma unroll
    for (int u = 0; u < UF; ++u) {
        const int blk = warp + u * W;
        float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = c0;
        if (blk < p.B * p.nb) {
            const float* y = p.gamma + (blk % p.nb) * QK + 8 * lane;
            c0 = ldg_f4_keep(y, keep);
            c1 = ldg_f4_keep(y + 4, keep);
        }
        gp[u][0] = c0.x; gp[u][1] = c0.y; gp[u][2] = c0.z; gp[u][3] = c0.w;
        gp[u][4] = c1.x; gp[u][5] = c1.y; gp[u][6] = c1.z; gp[u][7] = c1.w;
    }
}

// top_up(): called once by every warp after its first round of global loads
// is issued (the warp's remaining weight copies go out behind them).
template <int FOLD, int SRC, int W, bool LL, class TopUp>
__device__ void stage_activations(const MatvecParams& p, uint8_t* act, double* red, int ctid,
                                  const float (&gp)[STAGE_UF][8], uint32_t gen_in, TopUp&& top_up) {
    const int warp = ctid >> 5, lane = ctid & 31;
    const int nblk = p.B * p.nb;
    // Each warp stages blocks warp, warp+W, ...; U blocks at a time with all
    // their global loads issued before any is used, so the latency of the
    // (just produced, L2-resident) activations is paid once per U blocks.
    constexpr int U = 4;
    if (SRC == ACT_Q8K) {
        for (int blk0 = warp; blk0 < nblk; blk0 += W * U) {
            uint32_t w0[U], w1[U], bw[U];
            float dv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int blk = blk0 + u * W;
                w0[u] = w1[u] = bw[u] = 0;
                dv[u] = 0.f;
                if (blk < nblk) {
                    const uint8_t* src = p.xq + (int64_t)blk * Q8K_BYTES;
                    const uint32_t* qw = reinterpret_cast<const uint32_t*>(src + 4);
                    w0[u] = qw[2 * lane];
                    w1[u] = qw[2 * lane + 1];
                    if (lane == 0) dv[u] = *reinterpret_cast<const float*>(src);
                    if (lane < 8) bw[u] = *reinterpret_cast<const uint32_t*>(src + 260 + 4 * lane);
                }
            }
            if (blk0 == warp) top_up();
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int blk = blk0 + u * W;
                if (blk >= nblk) break;
                uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int wi = 2 * lane + h;
                    const uint32_t w = h ? w1[u] : w0[u];
                    if (FOLD == BH_FOLD_X86) {
                        *reinterpret_cast<uint32_t*>(dst + staged_byte_offset<FOLD>(4 * wi)) = w;
                    } else {
#pragma unroll
                        for (int b = 0; b < 4; ++b) dst[staged_byte_offset<FOLD>(4 * wi + b)] = (uint8_t)(w >> (8 * b));
                    }
                }
                if (lane == 0) *reinterpret_cast<float*>(dst + ACT_D_OFF) = dv[u];
                if (lane < 8) {
                    const int s = (int)(int16_t)(bw[u] & 0xffffu) + (int)(int16_t)(bw[u] >> 16);
                    reinterpret_cast<int16_t*>(dst + ACT_S_OFF)[lane] = (int16_t)s;
                }
            }
        }
        top_up();  // (no-op for warps that already did)
        return;
    }
    // fp32 sources. RMSNorm follows rms_norm_f32 (ggml-cpu/ops.cpp): every
    // square is a binary32 product, the squares are summed in double,
    // mean = (float)(sum / K), scale = 1 / sqrtf(mean + eps), x * scale, then
    // the norm weight (ggml_mul). The reference sums sequentially; here the
    // double sum runs as a tree, which changes the double result only in its
    // last bits and the binary32 mean only when the sum lies within that of a
    // binary32 rounding boundary. When every warp's blocks fit one round
    // (nblk <= W*UF, the decode shapes), all global loads are issued at once
    // and the sum of squares is taken from the loaded registers: per block
    // (lane sums in element order, then an xor butterfly), per column (the
    // blocks' sums through shared memory, one per lane, then an xor
    // butterfly, in every warp). The order is fixed, so every warp of every
    // CTA derives the same scale. Larger batches fall back to a separate
    // strided pass for the sum of squares.
    constexpr int UF = stage_uf<SRC>();
    __shared__ float s_scale[BH_MAX_BATCH];
    const bool one_round = nblk <= W * UF;
    auto rms_scale = [&](double sum) {
        const float mean = __double2float_rn(div_by_count(sum, p.K));
        return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    };
    if (SRC == ACT_F32_RMSNORM && !one_round) {
        for (int b = 0; b < p.B; ++b) {
            const float* h = p.xf + (int64_t)b * p.K;
            double ss = 0.0;
#pragma unroll 4
            for (int i = ctid; i < p.K; i += W * 32) ss = __dadd_rn(ss, (double)__fmul_rn(h[i], h[i]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if (lane == 0) red[warp] = ss;
            named_bar(1, W * 32);
            if (ctid == 0) {
                double t = 0.0;
                for (int w = 0; w < W; ++w) t = __dadd_rn(t, red[w]);
                s_scale[b] = rms_scale(t);
            }
            named_bar(1, W * 32);
        }
    }
    // every warp runs the same number of rounds (the RMSNorm path has CTA
    // barriers inside a round)
    const int rounds = (nblk + W * UF - 1) / (W * UF);
    for (int rd = 0; rd < rounds; ++rd) {
        const int blk0 = warp + rd * W * UF;
        float v[UF][8], aux[UF][8];
#pragma unroll
        for (int u = 0; u < UF; ++u) {
            const int blk = blk0 + u * W;
            const int b = blk / p.nb, i = blk - b * p.nb;
            const int e0 = i * QK + 8 * lane;
#pragma unroll
            for (int t = 0; t < 8; ++t) { v[u][t] = 0.f; aux[u][t] = 0.f; }
            if (blk < nblk) {
                if constexpr (LL) {
                    // row split: the exchanged pairs of this generation (LL
                    // kernels read their fp32 input from p.xf only when
                    // ll.x is null: the first layer's embedding)
                    if (p.ll.x) {
                        if (!tp_load8(p.ll.x + (int64_t)b * p.K + e0, gen_in, v[u], p.status))
                            set_status(p.status, ST_TIMEOUT);
                    } else {
                        const float* x = p.xf + (int64_t)b * p.K + e0;
                        const float4 a0 = *reinterpret_cast<const float4*>(x), a1 = *reinterpret_cast<const float4*>(x + 4);
                        v[u][0] = a0.x; v[u][1] = a0.y; v[u][2] = a0.z; v[u][3] = a0.w;
                        v[u][4] = a1.x; v[u][5] = a1.y; v[u][6] = a1.z; v[u][7] = a1.w;
                    }
                } else {
                    const float* x = p.xf + (int64_t)b * p.K + e0;
                    const float4 a0 = *reinterpret_cast<const float4*>(x), a1 = *reinterpret_cast<const float4*>(x + 4);
                    v[u][0] = a0.x; v[u][1] = a0.y; v[u][2] = a0.z; v[u][3] = a0.w;
                    v[u][4] = a1.x; v[u][5] = a1.y; v[u][6] = a1.z; v[u][7] = a1.w;
                }
                if constexpr (SRC == ACT_F32_RMSNORM) {
                    if (one_round) {
#pragma unroll
                        for (int t = 0; t < 8; ++t) aux[u][t] = gp[u][t];
                    } else {
                        const float* y = p.gamma + e0;
                        const float4 c0 = *reinterpret_cast<const float4*>(y), c1 = *reinterpret_cast<const float4*>(y + 4);
                        aux[u][0] = c0.x; aux[u][1] = c0.y; aux[u][2] = c0.z; aux[u][3] = c0.w;
                        aux[u][4] = c1.x; aux[u][5] = c1.y; aux[u][6] = c1.z; aux[u][7] = c1.w;
                    }
                }
            }
        }
        float scale_u[UF];
        if (rd == 0) top_up();
        if (SRC == ACT_F32_RMSNORM && one_round) {
            // red[blk]: sum of squares of block blk (nblk <= W*UF entries)
#pragma unroll
            for (int u = 0; u < UF; ++u) {
                const int blk = blk0 + u * W;
                double ss = 0.0;
#pragma unroll
                for (int t = 0; t < 8; ++t) ss = __dadd_rn(ss, (double)__fmul_rn(v[u][t], v[u][t]));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
                if (lane == 0 && blk < nblk) red[blk] = ss;
            }
            BH_TRACE_AT(1);
            named_bar(1, W * 32);
            // every warp sums its blocks' columns itself: lane i takes block i
            // of the column (nb <= 32 here), then an xor butterfly
#pragma unroll
            for (int u = 0; u < UF; ++u) {
                const int blk = blk0 + u * W;
                const int b = (blk < nblk ? blk : 0) / p.nb;
                double t = lane < p.nb ? red[b * p.nb + lane] : 0.0;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) t = __dadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
                scale_u[u] = rms_scale(t);
            }
        }
        auto quantize_block = [&](int u) {
            const int blk = blk0 + u * W;
            const int b = (blk < nblk ? blk : 0) / p.nb;
            float x[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (SRC == ACT_F32_RMSNORM) {
                    x[t] = __fmul_rn(__fmul_rn(v[u][t], one_round ? scale_u[u] : s_scale[b]), aux[u][t]);
                } else {
                    x[t] = v[u][t];
                }
            }
            const Q8Block qb = q8k_quantize_warp(x, lane);
            if (blk < nblk) {  // warp-uniform
                uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
                stage_codes<FOLD>(dst, qb.q, lane);
                stage_scalars(dst, qb.d, qb.bsum16, lane);
            }
        };
        if (nblk <= W) {
            quantize_block(0);  // one block per warp (the decode step's K = 4096 launches)
        } else {
            // every u is worked, so the UF quantize chains can interleave;
            // blocks past nblk are zeros and are not stored
#pragma unroll
            for (int u = 0; u < UF; ++u) quantize_block(u);
        }
        if (rd == 0) BH_TRACE_AT(7);
    }
    top_up();  // (no-op after the first round's call)
}

// Per-row epilogue of the dense kernel.
template <int FOLD, int EPI, int TPR, bool LL>
__device__ __forceinline__ void finish_row(const MatvecParams& p, const float (&acc)[RowBlk<TPR>::L], float accm, int rgrp,
                                           int t, int b, bool has_row, int64_t row, float& best_v, int& best_i,
                                           uint32_t gen_out) {
    const float v = row_value<FOLD, TPR>(acc, accm, rgrp);
    if (has_row && t == 0) {
        const int64_t yi = (int64_t)b * p.ldy + row;
        if (LL && p.ll.y_self && EPI != EPI_ARGMAX) {
            // row split: the pair into every rank's copy (the residual is
            // this rank's own row of the previous generation)
            const float hv = EPI == EPI_ADD ? __fadd_rn(__uint_as_float((uint32_t)p.ll.y_self[yi]), v) : v;
            tp_store(p.ll, yi, hv, gen_out);
        } else if (EPI == EPI_ADD) {
            float* yp = p.y + yi;
            const float hv = __fadd_rn(*yp, v);  // ggml_add(x, W.a)
            *yp = hv;
            if (p.capture) p.capture[yi] = hv;
        } else if (EPI != EPI_ARGMAX || p.y) {
            p.y[yi] = v;
        }
        if (EPI == EPI_ARGMAX && v > best_v) { best_v = v; best_i = (int)row; }
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Work is dealt in tiles of R = 32 / TPR consecutive rows of the CTA's
// range: warp w takes tiles w, w+8, ... and streams them through its own
// ring of `stages` stages. A stage is the next kc super-blocks of the
// tile's R rows, one 2-D tensor copy (box = R rows x row_stride bytes,
// rows padded so reads are bank-conflict free) issued by lane 0 and counted
// on the stage's mbarrier; the warp both fills and drains its ring (no
// cross-warp handshake). Thread (r, t) works row r of the tile; its fp32
// fold runs in registers as the blocks stream by.
template <int FOLD, int NB, int SRC, int EPI, bool PART, int TPR, bool LL>
__global__ void __launch_bounds__(dense_warps(NB, TPR) * 32, dense_min_blocks(NB, TPR)) q4k_matvec_kernel(const __grid_constant__ MatvecParams p) {
    constexpr int W = dense_warps(NB, TPR);
    constexpr int R = 32 / TPR;
    constexpr int L = RowBlk<TPR>::L;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[DENSE_MAX_WARPS];
    __shared__ int s_redi[DENSE_MAX_WARPS];
    __shared__ double s_ssq[DENSE_MAX_WARPS * STAGE_UF];  // RMSNorm: per-block (or per-warp) sums of squares
    BH_TRACE_AT(0);

    uint8_t* act = smem + p.act_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float gpre[STAGE_UF][8];
    if (SRC == ACT_F32_RMSNORM) preload_gamma<W>(p, gpre, warp, lane);
    uint8_t* ring = smem + p.ring_off + (size_t)warp * p.stages * p.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off) + warp * p.stages;

    // CTA ranges are whole tiles of the virtual matrix
    const int64_t ntile_all = (p.N + R - 1) / R;
    const int64_t r_begin = R * (ntile_all * blockIdx.x / gridDim.x);
    const int64_t r_end_t = R * (ntile_all * (blockIdx.x + 1) / gridDim.x);
    const int64_t r_end = r_end_t < p.N ? r_end_t : p.N;
    const int nrows = (int)(r_end - r_begin);
    const int ntiles = (nrows + R - 1) / R;
    const int my_tiles = warp < ntiles ? (ntiles - 1 - warp) / W + 1 : 0;
    const int nkc = (p.nb + p.kc - 1) / p.kc;
    const int total = my_tiles * nkc;
    const unsigned FULLM = 0xffffffffu;

    // (warps without a tile own no ring: the planner sized the rings for the
    // warps that have one)
    if (lane == 0 && my_tiles > 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const uint64_t pol = policy_evict_first();
    // issue cursor: (tile, chunk, stage), advanced without divisions; one
    // tensor-map box per stage (bytes past a row's end and rows past the
    // matrix are zero-filled and never used)
    int i_j = 0, i_c = 0, i_s = 0, issued = 0;
    auto issue_next = [&]() {
        if (lane == 0) {
            const int x = i_c * p.kc * (Q4K_BYTES / 8);
            uint8_t* dst = ring + (size_t)i_s * p.stage_bytes;
            mbar_arrive_expect_tx(&full[i_s], (uint32_t)(R * p.row_stride));  // one box (the stage may be padded)
            if (EPI == EPI_SWIGLU) {
                // one 3-D copy: R/2 gate rows, then the same R/2 up rows
                const int row = (int)((r_begin + (int64_t)(warp + i_j * W) * R) / 2);
                tensor_g2s_3d(dst, &p.tmap[0], x, row, 0, &full[i_s], pol);
            } else {
                int64_t local;
                const int sg = seg_of(p, r_begin + (int64_t)(warp + i_j * W) * R, local);
                tensor_g2s_2d(dst, &p.tmap[sg], x, (int)local, &full[i_s], pol);
            }
        }
        __syncwarp();
        ++issued;
        if (++i_c == nkc) { i_c = 0; ++i_j; }
        if (++i_s == p.stages) i_s = 0;
    };
    // weights do not depend on the previous kernel: the first p.prefill
    // stages of the ring go out now, the rest right behind the activation
    // loads after the wait (so those loads do not queue behind a full ring)
    const int ring_fill = min(p.stages, total);
    const int prefill = p.prefill > 0 ? min(p.prefill, ring_fill) : (p.prefill < 0 ? 0 : ring_fill);
    for (int q = 0; q < prefill; ++q) issue_next();
    pdl_trigger();
    pdl_wait();
    BH_TRACE_AT(5);
    // row split: generations of the exchanged input and output (the step
    // counter is final once the previous kernel has completed)
    const uint32_t gen_in = LL && p.ll.x ? tp_gen(p.ll, p.ll.gen_in) : 0u;
    const uint32_t gen_out = LL && p.ll.y_self ? tp_gen(p.ll, p.ll.gen_out) : 0u;
    // this warp's share of the L2 prefetch of a later launch's weights: now
    // when it has no copies of its own, else right after its last copy
    const int64_t wg = (int64_t)blockIdx.x * W + warp, nwg = (int64_t)gridDim.x * W;
    bool prefetched = false;
    if (total == 0) {
        prefetch_share(p.pf_ptr, p.pf_bytes, wg, nwg, lane);
        prefetched = true;
    }
    stage_activations<FOLD, SRC, W, LL>(p, act, s_ssq, threadIdx.x, gpre, gen_in, [&]() {
        while (issued < ring_fill) issue_next();
    });
    __syncthreads();
    BH_TRACE_AT(2);

    const int rgrp = lane / TPR;  // row of the tile worked by this thread
    const int t = lane % TPR;

    float best_v[NB];
    int best_i[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { best_v[b] = -INFINITY; best_i[b] = 0x7fffffff; }

    int consumed = 0, c_s = 0;
    uint32_t c_ph = 0;
    bool ok = true;
    for (int j = 0; j < my_tiles && ok; ++j) {
        const int rin = (warp + j * W) * R + rgrp;
        const bool live = rin < nrows;
        float acc[NB][L], accm[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int e = 0; e < L; ++e) acc[b][e] = 0.f;
            accm[b] = 0.f;
        }
        for (int c = 0; c < nkc; ++c) {
            if (!__all_sync(FULLM, mbar_wait_bounded(&full[c_s], c_ph))) {
                ok = false;
                if (lane == 0) set_status(p.status, ST_TIMEOUT);
                break;
            }
#ifdef BH_TRACE
            if (consumed == 0) BH_TRACE_AT(3);
#endif
            ++consumed;
            const int sbc = c * p.kc;
            const int kl = min(p.kc, p.nb - sbc);
            // rows past the end of the range read zero-filled stage bytes and are never stored
            const uint8_t* rowp = ring + (size_t)c_s * p.stage_bytes + (size_t)rgrp * p.row_stride;
            const uint8_t* actc = act + sbc * ACT_BLOCK_BYTES;
BH_UNROLL(BH_KB_UNROLL)
            for (int kb = 0; kb < kl; ++kb) {
                const RowBlk<TPR> r = decode_row<FOLD, TPR>(rowp + kb * Q4K_BYTES, t);
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    fold_block<FOLD, PART, TPR>(
                        r, actc + (b * p.nb + kb) * ACT_BLOCK_BYTES, t,
                        PART && live ? p.partials + (((int64_t)b * p.N + r_begin + rin) * p.nb + sbc + kb) * 9 : nullptr,
                        acc[b], accm[b]);
            }
            __syncwarp();
            if (issued < total) {
                fence_proxy_async_smem();
                issue_next();
            } else if (!prefetched) {
                prefetch_share(p.pf_ptr, p.pf_bytes, wg, nwg, lane);
                prefetched = true;
            }
            if (++c_s == p.stages) { c_s = 0; c_ph ^= 1u; }
        }
        if (!ok) break;
        BH_TRACE_AT(4);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (EPI == EPI_SWIGLU) {
                // gate row i in row group rgrp < R/2, its up row R/2 groups
                // (16 lanes) further on
                const float v = row_value<FOLD, TPR>(acc[b], accm[b], rgrp);
                const float u = __shfl_down_sync(FULLM, v, 16);
                if (live && t == 0 && rgrp < R / 2) {
                    const int64_t i = (r_begin + (int64_t)(warp + j * W) * R) / 2 + rgrp;
                    const float a = __fmul_rn(silu_ggml(v), u);  // ggml_silu then ggml_mul
                    if (LL && p.ll.y_self)
                        tp_store(p.ll, (int64_t)b * p.ldy + i, a, gen_out);
                    else
                        p.y[(int64_t)b * p.ldy + i] = a;
                    if (p.capture) {  // the gate and up rows before the SwiGLU
                        p.capture[(int64_t)b * 2 * p.ldy + i] = v;
                        p.capture[(int64_t)b * 2 * p.ldy + p.ldy + i] = u;
                    }
                }
            } else {
                finish_row<FOLD, EPI, TPR, LL>(p, acc[b], accm[b], rgrp, t, b, live, r_begin + rin, best_v[b], best_i[b],
                                           gen_out);
            }
        }
    }
    BH_TRACE_AT(6);
    if (!ok && lane == 0) {
        // nothing of this warp may still be in flight when the CTA exits
        int s = c_s;
        uint32_t ph = c_ph;
        for (int q = consumed; q < issued; ++q) {
            mbar_wait_bounded(&full[s], ph);
            if (++s == p.stages) { s = 0; ph ^= 1u; }
        }
    }

    if (EPI == EPI_ARGMAX) {
        // CTA candidates: maximum value, first index among equals
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float bv = best_v[b];
            int bi = best_i[b];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(FULLM, bv, off);
                const int oi = __shfl_xor_sync(FULLM, bi, off);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) { s_red[warp] = bv; s_redi[warp] = bi; }
            __syncthreads();
            if (threadIdx.x == 0) {
                float cv = s_red[0];
                int ci = s_redi[0];
                for (int w = 1; w < W; ++w)
                    if (s_red[w] > cv || (s_red[w] == cv && s_redi[w] < ci)) { cv = s_red[w]; ci = s_redi[w]; }
                p.cand_val[blockIdx.x * p.B + b] = cv;
                p.cand_idx[blockIdx.x * p.B + b] = ci;
            }
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Plan one launch: R = 32 / tpr rows per stage, kc super-blocks per row per
// stage (from the copy target, shrunk until 2 stages fit; box rows stay
// within 2048 bytes), 2-8 stages. Only the warps that own a tile get a ring
// (a CTA's range is at most ceil(tiles / grid) tiles), so a matrix with few
// rows per CTA gives its working warps deeper rings, which fill before the
// programmatic wait.
int matvec_plan(MatvecParams& p, int grid, int smem_cap, int stage_target, int tpr) {
    if (grid < 1 || (tpr != 4 && tpr != 8 && tpr != 16)) return BH_EINVAL;
    const int R = 32 / tpr;
    const int W = dense_warps(p.B, tpr);
    const int64_t tiles_cta = ((p.N + R - 1) / R + grid - 1) / grid;
    const int wbusy = tiles_cta < W ? (int)(tiles_cta > 0 ? tiles_cta : 1) : W;
    const int act_bytes = p.B * p.nb * ACT_BLOCK_BYTES;
    const int ring_off = (act_bytes + 127) / 128 * 128;
    int kc = stage_target / Q4K_BYTES;
    if (kc < 1) kc = 1;
    if (kc > 13) kc = 13;  // box rows of at most 2048 bytes (256 eight-byte elements)
    if (kc > p.nb) kc = p.nb;
    for (; kc >= 1; --kc) {
        const int words = kc * (Q4K_BYTES / 4);
        const int padw = ((8 - (words % 32)) % 32 + 32) % 32;  // row stride == 8 words (mod 32 banks)
        const int stride = kc * Q4K_BYTES + 4 * padw;
        // (stride is 32 mod 128 bytes, so R * stride, R = 4 or 8, is a
        // multiple of 128; two-row stages are padded to one: every stage
        // starts 128-byte aligned, as a tensor copy's shared-memory
        // destination must)
        const int stage = (R * stride + 127) / 128 * 128;
        const int avail = smem_cap - ring_off - 512;  // static shared memory of the kernel
        int stages = avail > 0 ? avail / (wbusy * (stage + 8)) : 0;
        if (stages > 8) stages = 8;
        if (stages < 2) continue;
        p.kc = kc;
        p.row_stride = stride;
        p.stage_bytes = stage;
        p.stages = stages;
        p.rows_per_tile = R;
        p.tpr = tpr;
        p.act_off = 0;
        p.ring_off = ring_off;
        p.bar_off = ring_off + wbusy * stages * stage;
        p.smem_bytes = p.bar_off + wbusy * stages * 8;
        return BH_OK;
    }
    return BH_EINVAL;  // activations too large for shared memory
}

template <int FOLD, int NB, int SRC, int EPI, bool PART, int TPR, bool LL = false>
static int launch_t(const MatvecParams& p, const LaunchOpts& o, int grid) {
    auto kern = q4k_matvec_kernel<FOLD, NB, SRC, EPI, PART, TPR, LL>;
    static std::atomic<uint64_t> attr_devices{0};
    // all kernels of a step ask for the same (largest) shared-memory
    // carveout, so consecutive launches can share an SM without the SM
    // having to drain and reconfigure between them
    if (!attrs_on_device(attr_devices, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
                       cudaSuccess &&
                   cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared) == cudaSuccess;
        }))
        return BH_EIO;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(dense_warps(NB, TPR) * 32);
    cfg.dynamicSmemBytes = (size_t)p.smem_bytes;
    cfg.stream = o.stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = o.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? BH_OK : BH_EIO;
}

template <int FOLD, int SRC, int EPI, bool PART>
static int launch_nb(const MatvecParams& p, const LaunchOpts& o, int grid) {
    if (p.tpr == 16) {
        // sixteen threads per row: matrices with at most 2 rows per warp, batch <= 2, x86 fold
        if constexpr (FOLD == BH_FOLD_X86 && !PART) {
            switch (p.B) {
                case 1: return launch_t<FOLD, 1, SRC, EPI, PART, 16>(p, o, grid);
                case 2: return launch_t<FOLD, 2, SRC, EPI, PART, 16>(p, o, grid);
                default: return BH_EINVAL;
            }
        }
        return BH_EINVAL;
    }
    if (p.tpr == 8) {
        // eight threads per row, 16-warp CTAs: narrow matrices
        switch (p.B) {
            case 1: return launch_t<FOLD, 1, SRC, EPI, PART, 8>(p, o, grid);
            case 2: return launch_t<FOLD, 2, SRC, EPI, PART, 8>(p, o, grid);
            case 3: return launch_t<FOLD, 3, SRC, EPI, PART, 8>(p, o, grid);
            case 4: return launch_t<FOLD, 4, SRC, EPI, PART, 8>(p, o, grid);
            case 5: return launch_t<FOLD, 5, SRC, EPI, PART, 8>(p, o, grid);
            case 6: return launch_t<FOLD, 6, SRC, EPI, PART, 8>(p, o, grid);
            case 7: return launch_t<FOLD, 7, SRC, EPI, PART, 8>(p, o, grid);
            case 8: return launch_t<FOLD, 8, SRC, EPI, PART, 8>(p, o, grid);
            default: return BH_EINVAL;
        }
    }
    switch (p.B) {
        case 1: return launch_t<FOLD, 1, SRC, EPI, PART, 4>(p, o, grid);
        case 2: return launch_t<FOLD, 2, SRC, EPI, PART, 4>(p, o, grid);
        case 3: return launch_t<FOLD, 3, SRC, EPI, PART, 4>(p, o, grid);
        case 4: return launch_t<FOLD, 4, SRC, EPI, PART, 4>(p, o, grid);
        case 5: return launch_t<FOLD, 5, SRC, EPI, PART, 4>(p, o, grid);
        case 6: return launch_t<FOLD, 6, SRC, EPI, PART, 4>(p, o, grid);
        case 7: return launch_t<FOLD, 7, SRC, EPI, PART, 4>(p, o, grid);
        case 8: return launch_t<FOLD, 8, SRC, EPI, PART, 4>(p, o, grid);
        default: return BH_EINVAL;
    }
}

// Row-split launches (exchanged pairs in or out): batch 1, the x86 fold, no
// partials; their own instantiations, so that one GPU's kernels carry none of
// the pair code (measured: it cost the one-GPU step 1.667 -> 1.746 ms).
template <int SRC, int EPI>
static int launch_ll_tpr(const MatvecParams& p, const LaunchOpts& o, int grid) {
    if (p.tpr == 8) return launch_t<BH_FOLD_X86, 1, SRC, EPI, false, 8, true>(p, o, grid);
    if (p.tpr == 4) return launch_t<BH_FOLD_X86, 1, SRC, EPI, false, 4, true>(p, o, grid);
    return BH_EINVAL;
}

static int launch_ll(const MatvecParams& p, int src, int epi, const LaunchOpts& o, int grid) {
    if (p.B != 1 || p.partials) return BH_EINVAL;
    switch (src * 4 + epi) {
        case ACT_F32 * 4 + EPI_ADD: return launch_ll_tpr<ACT_F32, EPI_ADD>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_STORE: return launch_ll_tpr<ACT_F32_RMSNORM, EPI_STORE>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_SWIGLU: return launch_ll_tpr<ACT_F32_RMSNORM, EPI_SWIGLU>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_ARGMAX: return launch_ll_tpr<ACT_F32_RMSNORM, EPI_ARGMAX>(p, o, grid);
        default: return BH_EINVAL;
    }
}

template <int FOLD>
static int launch_fold(const MatvecParams& p, int src, int epi, const LaunchOpts& o, int grid) {
    const bool part = p.partials != nullptr;
    if (part) {
        if (src != ACT_Q8K || epi != EPI_STORE) return BH_EINVAL;
        return launch_nb<FOLD, ACT_Q8K, EPI_STORE, true>(p, o, grid);
    }
    switch (src * 4 + epi) {
        case ACT_Q8K * 4 + EPI_STORE: return launch_nb<FOLD, ACT_Q8K, EPI_STORE, false>(p, o, grid);
        case ACT_Q8K * 4 + EPI_ARGMAX: return launch_nb<FOLD, ACT_Q8K, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32 * 4 + EPI_STORE: return launch_nb<FOLD, ACT_F32, EPI_STORE, false>(p, o, grid);
        case ACT_F32 * 4 + EPI_ADD: return launch_nb<FOLD, ACT_F32, EPI_ADD, false>(p, o, grid);
        case ACT_F32 * 4 + EPI_ARGMAX: return launch_nb<FOLD, ACT_F32, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_STORE: return launch_nb<FOLD, ACT_F32_RMSNORM, EPI_STORE, false>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_ARGMAX: return launch_nb<FOLD, ACT_F32_RMSNORM, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32_RMSNORM * 4 + EPI_SWIGLU: return launch_nb<FOLD, ACT_F32_RMSNORM, EPI_SWIGLU, false>(p, o, grid);
        default: return BH_EINVAL;
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        cudaGetLastError();
    }
    return fn;
}

// A 2-D tensor map over a Q4_K matrix: 8-byte elements, rows of nb*144
// bytes, `rows` high; the box is box_rows rows x row_stride bytes.
int encode_q4k_map(CUtensorMap* map, const void* base, int64_t rows, int nb, int row_stride, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return BH_EIO;
    const int64_t rowbytes = (int64_t)nb * Q4K_BYTES;
    const cuuint64_t dims[2] = {(cuuint64_t)(rowbytes / 8), (cuuint64_t)(rows > 0 ? rows : 1)};
    const cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
    const cuuint32_t box[2] = {(cuuint32_t)(row_stride / 8), (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return BH_EINVAL;
    return BH_OK;
}

// A 3-D tensor map over a gate matrix and the up matrix `dist` bytes after it
// (both `rows` x nb*144 bytes): box = row_stride bytes x box_rows rows x 2.
int encode_q4k_pair_map(CUtensorMap* map, const void* gate, int64_t rows, int nb, int64_t dist, int row_stride,
                        int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return BH_EIO;
    const int64_t rowbytes = (int64_t)nb * Q4K_BYTES;
    const cuuint64_t dims[3] = {(cuuint64_t)(rowbytes / 8), (cuuint64_t)(rows > 0 ? rows : 1), 2};
    const cuuint64_t strides[2] = {(cuuint64_t)rowbytes, (cuuint64_t)dist};
    const cuuint32_t box[3] = {(cuuint32_t)(row_stride / 8), (cuuint32_t)box_rows, 2};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(gate), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return BH_EINVAL;
    return BH_OK;
}

// One tensor map per segment; the box is the stage slice of one tile. Gate/up
// pairs (two segments of `half` rows each) use one 3-D map over both
// matrices: x = 8-byte element of a row, y = row, z = matrix (stride: the
// distance from the gate to the up matrix); a box of R/2 rows x 2 matrices
// lands as the R/2 gate rows followed by the same R/2 up rows.
static int encode_maps(MatvecParams& p, bool pair) {
    if (pair) {
        const int64_t half = p.seg_end[0];
        const int64_t rowbytes = (int64_t)p.nb * Q4K_BYTES;
        const int64_t dist = p.w[1] - p.w[0];
        if (2 * half != p.N || p.seg_end[1] != p.N || half % (p.rows_per_tile / 2)) return BH_EINVAL;
        if (dist < half * rowbytes || dist % 16) return BH_EINVAL;  // up after gate, no overlap
        return encode_q4k_pair_map(&p.tmap[0], p.w[0], half, p.nb, dist, p.row_stride, p.rows_per_tile / 2);
    }
    if (p.seg_end[0] < p.N && (p.seg_end[0] % MV_ROWS || p.seg_end[1] % MV_ROWS)) return BH_EINVAL;
    int64_t prev = 0;
    for (int sg = 0; sg < 3; ++sg) {
        const int64_t rows = p.seg_end[sg] - prev;
        prev = p.seg_end[sg];
        const int rc = encode_q4k_map(&p.tmap[sg], p.w[sg], rows, p.nb, p.row_stride, p.rows_per_tile);
        if (rc != BH_OK) return rc;
    }
    return BH_OK;
}

int launch_matvec(const MatvecParams& pin, int fold, int act_src, int epi, const LaunchOpts& o) {
    MatvecParams p = pin;
    // a tensor copy's shared-memory destination must be 128-byte aligned
    if (p.stage_bytes % 128 || (epi == EPI_SWIGLU && p.partials)) return BH_EINVAL;
    const int rc = encode_maps(p, epi == EPI_SWIGLU);
    if (rc != BH_OK) return rc;
    const int grid = o.grid;
    if (p.ll.x || p.ll.y_self) return fold == BH_FOLD_X86 ? launch_ll(p, act_src, epi, o, grid) : BH_EINVAL;
    if (fold == BH_FOLD_X86) return launch_fold<BH_FOLD_X86>(p, act_src, epi, o, grid);
    if (fold == BH_FOLD_GENERIC) return launch_fold<BH_FOLD_GENERIC>(p, act_src, epi, o, grid);
    return BH_EINVAL;
}

}  // namespace bh
