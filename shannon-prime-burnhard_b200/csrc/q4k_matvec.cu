// q4k_matvec.cu — the sm_100a Q4_K x Q8_K matvec (batch 1..8).
//
// Structure (one CTA of 8 warps per SM, persistent over a contiguous range
// of rows):
//  - every warp owns "quads" of 4 consecutive rows and streams them through
//    its own ring of shared-memory stages with 1-D bulk async copies
//    (cp.async.bulk, the TMA engine), completion counted on per-stage
//    mbarriers; one copy per row per stage, rows padded so reads are
//    bank-conflict free. Eight warps issue copies in parallel (a single
//    issuing warp caps small-copy throughput far below HBM bandwidth).
//    Weights do not depend on the previous kernel, so each warp starts
//    streaming before the programmatic-launch wait.
//  - all warps stage the activations once (Q8_K input, or fp32
//    input quantized in the prologue), then each row is worked by 8 threads:
//    thread "lane" j of the row owns exactly the int32 lane j of the
//    reference's vec_dot, so its fp32 fold chain stays in registers and the
//    result is bit-identical to the reference's fold:
//      FOLD_X86     (ggml-cpu/arch/x86/quants.c:1900-1983): lane m = bytes
//                   4m..4m+3 of every 32-byte quant group -> a natural word,
//                   one dp4a per nibble half; acc = fma(d, sumi, acc).
//      FOLD_GENERIC (ggml-cpu/quants.c:645-718): lane l = positions p % 8 == l,
//                   a 4x4 byte transpose (prmt) per word; sums += d * aux.
//    Integer sums are exact (|partial| < 2^24), so only the fp32 order
//    matters, and it is reproduced operation by operation.
#include "bh_common.cuh"
#include "bh_kernels.cuh"
#include "q8k_device.cuh"

namespace bh {

__device__ __forceinline__ const uint8_t* seg_row(const MatvecParams& p, int64_t row) {
    const int64_t rowb = (int64_t)p.nb * Q4K_BYTES;
    if (row < p.seg_end[0]) return p.w[0] + row * rowb;
    if (row < p.seg_end[1]) return p.w[1] + (row - p.seg_end[0]) * rowb;
    return p.w[2] + (row - p.seg_end[1]) * rowb;
}

// ---------------------------------------------------------------------------
// prologue: activations -> staged Q8_K blocks in shared memory
// ---------------------------------------------------------------------------
template <int FOLD, int SRC>
__device__ void stage_activations(const MatvecParams& p, uint8_t* act, float* red, int ctid) {
    const int warp = ctid >> 5, lane = ctid & 31;
    const int nblk = p.B * p.nb;
    if (SRC == ACT_Q8K) {
        for (int blk = warp; blk < nblk; blk += MV_WARPS) {
            const uint8_t* src = p.xq + (int64_t)blk * Q8K_BYTES;
            uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
            const uint32_t* qw = reinterpret_cast<const uint32_t*>(src + 4);
            if (FOLD == BH_FOLD_X86) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int wi = 2 * lane + h;
                    *reinterpret_cast<uint32_t*>(dst + staged_byte_offset<FOLD>(4 * wi)) = qw[wi];
                }
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int wi = 2 * lane + h;
                    const uint32_t w = qw[wi];
#pragma unroll
                    for (int b = 0; b < 4; ++b) dst[staged_byte_offset<FOLD>(4 * wi + b)] = (uint8_t)(w >> (8 * b));
                }
            }
            if (lane == 0) *reinterpret_cast<float*>(dst + 256) = *reinterpret_cast<const float*>(src);
            if (lane < 8) {
                const uint32_t bw = *reinterpret_cast<const uint32_t*>(src + 260 + 4 * lane);
                const int s = (int)(int16_t)(bw & 0xffffu) + (int)(int16_t)(bw >> 16);
                reinterpret_cast<int16_t*>(dst + 272)[lane] = (int16_t)s;
            }
        }
        return;
    }
    // fp32 sources
    __shared__ float s_scale[BH_MAX_BATCH];
    if (SRC == ACT_F32_RMSNORM) {
        // fixed-order reduction, identical in every CTA
        for (int b = 0; b < p.B; ++b) {
            const float* h = p.xf + (int64_t)b * p.K;
            float ss = 0.f;
            for (int i = ctid; i < p.K; i += MV_WARPS * 32) ss = __fadd_rn(ss, __fmul_rn(h[i], h[i]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if (lane == 0) red[warp] = ss;
            named_bar(1, MV_WARPS * 32);
            if (ctid == 0) {
                float t = 0.f;
                for (int w = 0; w < MV_WARPS; ++w) t = __fadd_rn(t, red[w]);
                const float mean = __fdiv_rn(t, (float)p.K);
                s_scale[b] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            }
            named_bar(1, MV_WARPS * 32);
        }
    }
    for (int blk = warp; blk < nblk; blk += MV_WARPS) {
        const int b = blk / p.nb, i = blk - b * p.nb;
        const int e0 = i * QK + 8 * lane;
        float v[8];
        if (SRC == ACT_F32_SWIGLU) {
            const float* g = p.xf + (int64_t)b * 2 * p.K + e0;
            const float* u = g + p.K;
            const float4 g0 = *reinterpret_cast<const float4*>(g), g1 = *reinterpret_cast<const float4*>(g + 4);
            const float4 u0 = *reinterpret_cast<const float4*>(u), u1 = *reinterpret_cast<const float4*>(u + 4);
            const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float sg = __fdiv_rn(gv[t], __fadd_rn(1.f, expf(-gv[t])));
                v[t] = __fmul_rn(sg, uv[t]);
            }
        } else {
            const float* x = p.xf + (int64_t)b * p.K + e0;
            const float4 a0 = *reinterpret_cast<const float4*>(x), a1 = *reinterpret_cast<const float4*>(x + 4);
            v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
            v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
            if (SRC == ACT_F32_RMSNORM) {
                const float sc = s_scale[b];
                const float4 c0 = *reinterpret_cast<const float4*>(p.gamma + e0);
                const float4 c1 = *reinterpret_cast<const float4*>(p.gamma + e0 + 4);
                const float gm[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(__fmul_rn(v[t], sc), gm[t]);
            }
        }
        const Q8Block qb = q8k_quantize_warp(v, lane);
        uint8_t* dst = act + blk * ACT_BLOCK_BYTES;
        stage_codes<FOLD>(dst, qb.q, lane);
        stage_scalars(dst, qb.d, qb.bsum16, lane);
    }
}

// ---------------------------------------------------------------------------
// per-super-block work of one thread (two reference lanes of one row)
// ---------------------------------------------------------------------------
// Thread t (0..3) of a row owns reference lanes 2t and 2t+1. Row side of
// one super-block: the two fp16 scales, the packed 6-bit scales/mins, and
// the low/high-nibble code words of both lanes.
struct RowBlk {
    float fd, fdm;
    uint32_t sc03, sc47, mnk;   // mnk: the two mins of min lane k = t in bytes 0..1
    uint32_t lo[2][4], hi[2][4];
};

template <int FOLD>
__device__ __forceinline__ RowBlk decode_row(const uint8_t* blk, int t) {
    RowBlk r;
    const uint4 h = *reinterpret_cast<const uint4*>(blk);
    r.fd = h2f((uint16_t)(h.x & 0xffffu));
    r.fdm = h2f((uint16_t)(h.x >> 16));
    // 6-bit scales/mins, get_scale_min_k4 (ggml-quants.c:818-825) word-wise:
    // j<4: sc = q[j] & 63, mn = q[j+4] & 63;
    // j>=4: sc = (q[j+4] & 15) | (q[j-4] >> 6) << 4, mn = (q[j+4] >> 4) | (q[j] >> 6) << 4
    r.sc03 = h.y & 0x3f3f3f3fu;
    r.sc47 = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn = (t & 2) ? (((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3f3f3f3fu);
    r.mnk = mn >> ((t & 1) * 16);
    const uint32_t* qs = reinterpret_cast<const uint32_t*>(blk + 16);
    if (FOLD == BH_FOLD_X86) {
        // lane m = bytes 4m..4m+3 of each 32-byte group: words 2t, 2t+1
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint2 w = *reinterpret_cast<const uint2*>(qs + 8 * g + 2 * t);
            r.lo[0][g] = w.x & 0x0f0f0f0fu;
            r.hi[0][g] = (w.x >> 4) & 0x0f0f0f0fu;
            r.lo[1][g] = w.y & 0x0f0f0f0fu;
            r.hi[1][g] = (w.y >> 4) & 0x0f0f0f0fu;
        }
    } else {
        // lane l = group bytes l, l+8, l+16, l+24 (a byte gather); lanes 2t and
        // 2t+1 sit in the same words k0 = t/2 + {0,2,4,6}, bytes tb and tb+1
        const int k0 = t >> 1, tb = (2 * t) & 3;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint32_t* gw = qs + 8 * g;
            const uint32_t w0 = gw[k0], w1 = gw[k0 + 2], w2 = gw[k0 + 4], w3 = gw[k0 + 6];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const uint32_t sel = (uint32_t)((tb + e) | ((tb + e + 4) << 4));
                const uint32_t tw = __byte_perm(__byte_perm(w0, w1, sel), __byte_perm(w2, w3, sel), 0x5410);
                r.lo[e][g] = tw & 0x0f0f0f0fu;
                r.hi[e][g] = (tw >> 4) & 0x0f0f0f0fu;
            }
        }
    }
    return r;
}

// One lane's exact integer sum over the super-block:
// sum_j sc_j * (dot of its 4 codes of sub-block j). Each sub-block dot is a
// dp4a (|dot| <= 4*15*127, fits int16); two of them are packed and scaled by
// two 6-bit scales in one dp2a.
__device__ __forceinline__ int lane_sum(const uint32_t (&lo)[4], const uint32_t (&hi)[4], uint32_t sc03,
                                        uint32_t sc47, const int4 a0, const int4 a1, int (&sub)[8], bool want_sub) {
    const int d0 = dp4a((int)lo[0], a0.x, 0), d1 = dp4a((int)hi[0], a0.y, 0);
    const int d2 = dp4a((int)lo[1], a0.z, 0), d3 = dp4a((int)hi[1], a0.w, 0);
    const int d4 = dp4a((int)lo[2], a1.x, 0), d5 = dp4a((int)hi[2], a1.y, 0);
    const int d6 = dp4a((int)lo[3], a1.z, 0), d7 = dp4a((int)hi[3], a1.w, 0);
    if (want_sub) {
        sub[0] = d0; sub[1] = d1; sub[2] = d2; sub[3] = d3;
        sub[4] = d4; sub[5] = d5; sub[6] = d6; sub[7] = d7;
    }
    int s = __dp2a_lo((int)__byte_perm((uint32_t)d0, (uint32_t)d1, 0x5410), (int)sc03, 0);
    s = __dp2a_hi((int)__byte_perm((uint32_t)d2, (uint32_t)d3, 0x5410), (int)sc03, s);
    s = __dp2a_lo((int)__byte_perm((uint32_t)d4, (uint32_t)d5, 0x5410), (int)sc47, s);
    return __dp2a_hi((int)__byte_perm((uint32_t)d6, (uint32_t)d7, 0x5410), (int)sc47, s);
}

// One activation column applied to one decoded row block: the reference's
// per-block fp32 step for this thread's two lanes and its min lane.
template <int FOLD, bool PART>
__device__ __forceinline__ void fold_block(const MatvecParams& p, const RowBlk& r, const uint8_t* A, int t,
                                           int b, int i, int64_t row, bool live, float& acc0, float& acc1,
                                           float& accm) {
    const int4 a00 = *reinterpret_cast<const int4*>(A + 64 * t);
    const int4 a01 = *reinterpret_cast<const int4*>(A + 64 * t + 16);
    const int4 a10 = *reinterpret_cast<const int4*>(A + 64 * t + 32);
    const int4 a11 = *reinterpret_cast<const int4*>(A + 64 * t + 48);
    const float yd = *reinterpret_cast<const float*>(A + 256);
    int sub0[8], sub1[8];
    const int l0 = lane_sum(r.lo[0], r.hi[0], r.sc03, r.sc47, a00, a01, sub0, PART);
    const int l1 = lane_sum(r.lo[1], r.hi[1], r.sc03, r.sc47, a10, a11, sub1, PART);
    if (FOLD == BH_FOLD_X86) {
        // acc[m] = fma(y.d * fp16(d), sumi[m], acc[m]);
        // accm[k] = fma(-y.d * fp16(dmin), min_{2k} S_{2k} + min_{2k+1} S_{2k+1}, accm[k]), k = t
        const float d = __fmul_rn(yd, r.fd);
        acc0 = __fmaf_rn(d, i2f_exact(l0), acc0);
        acc1 = __fmaf_rn(d, i2f_exact(l1), acc1);
        const int spk = reinterpret_cast<const int*>(A + 272)[t];
        accm = __fmaf_rn(__fmul_rn(-yd, r.fdm), i2f_exact(__dp2a_lo(spk, (int)r.mnk, 0)), accm);
    } else {
        // sums[l] += (fp16(d) * y.d) * aux[l];  sumf -= (fp16(dmin) * y.d) * sumi
        const float d = __fmul_rn(r.fd, yd);
        acc0 = __fadd_rn(acc0, __fmul_rn(d, i2f_exact(l0)));
        acc1 = __fadd_rn(acc1, __fmul_rn(d, i2f_exact(l1)));
        // sumi = the four threads' min pairs (exact ints) summed in thread 0
        const int spk = reinterpret_cast<const int*>(A + 272)[t];
        int mp = __dp2a_lo(spk, (int)r.mnk, 0);
        mp += __shfl_xor_sync(0xffffffffu, mp, 1);
        mp += __shfl_xor_sync(0xffffffffu, mp, 2);
        accm = __fsub_rn(accm, __fmul_rn(__fmul_rn(r.fdm, yd), i2f_exact(mp)));
    }
    if (PART) {
        int mp = __dp2a_lo(reinterpret_cast<const int*>(A + 272)[t], (int)r.mnk, 0);
        mp += __shfl_xor_sync(0xffffffffu, mp, 1);
        mp += __shfl_xor_sync(0xffffffffu, mp, 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int v = sub0[j] + sub1[j];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            sub0[j] = v;
        }
        if (live && t == 0) {
            int32_t* o = p.partials + (((int64_t)b * p.N + row) * p.nb + i) * 9;
            for (int j = 0; j < 8; ++j) o[j] = sub0[j];
            o[8] = mp;
        }
    }
}

// Per-row combine in the reference's order, then the epilogue.
template <int FOLD, int EPI>
__device__ __forceinline__ void finish_row(const MatvecParams& p, float acc0, float acc1, float accm, int rgrp,
                                           int t, int b, bool has_row, int64_t row, float& best_v, int& best_i) {
    const unsigned FULLM = 0xffffffffu;
    float v;
    if (FOLD == BH_FOLD_X86) {
        // hsum_float_8 (arch/x86/quants.c:43-49): ((a4+a0)+(a6+a2)) + ((a5+a1)+(a7+a3));
        // thread t holds lanes 2t (acc0) and 2t+1 (acc1)
        const float x0 = __fadd_rn(acc0, __shfl_xor_sync(FULLM, acc0, 2));  // t0: a0+a4, t1: a2+a6
        const float x1 = __fadd_rn(acc1, __shfl_xor_sync(FULLM, acc1, 2));  // t0: a1+a5, t1: a3+a7
        const float y0 = __fadd_rn(x0, __shfl_xor_sync(FULLM, x0, 1));
        const float y1 = __fadd_rn(x1, __shfl_xor_sync(FULLM, x1, 1));
        const float hs = __fadd_rn(y0, y1);
        // 4-lane min accumulator, lane k in thread k: (m0+m2) + (m1+m3)
        const float u = __fadd_rn(accm, __shfl_xor_sync(FULLM, accm, 2));
        const float hm = __fadd_rn(u, __shfl_xor_sync(FULLM, u, 1));
        v = __fadd_rn(hs, hm);
    } else {
        // sumf (the min chain) += sums[0..7] in order
        v = accm;
#pragma unroll
        for (int l = 0; l < 8; ++l) v = __fadd_rn(v, __shfl_sync(FULLM, (l & 1) ? acc1 : acc0, (rgrp << 2) + (l >> 1)));
    }
    if (has_row && t == 0) {
        float* yp = p.y + (int64_t)b * p.ldy + row;
        if (EPI == EPI_ADD) *yp = __fadd_rn(*yp, v);
        else if (EPI != EPI_ARGMAX || p.y) *yp = v;
        if (EPI == EPI_ARGMAX && v > best_v) { best_v = v; best_i = (int)row; }
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Each warp owns "octs" of 8 consecutive rows (oct w, w+8, ... of the CTA's
// row range) and runs its own ring of `stages` stages: a stage is the next kc
// super-blocks of the oct's 8 rows, one bulk copy per row issued by lanes
// 0..7 and counted on the stage's mbarrier. Thread (r, t) works row r of the
// oct as reference lanes 2t and 2t+1 (and min lane t). The warp both fills
// and drains its ring: no cross-warp handshake, and eight warps issue copies
// in parallel.
template <int FOLD, int NB, int SRC, int EPI, bool PART>
__global__ void __launch_bounds__(MV_THREADS, 1) q4k_matvec_kernel(const MatvecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[MV_WARPS * 2];
    __shared__ int s_redi[MV_WARPS];

    uint8_t* act = smem + p.act_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = smem + p.ring_off + (size_t)warp * p.stages * p.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off) + warp * p.stages;

    const int64_t r_begin = p.N * blockIdx.x / gridDim.x;
    const int64_t r_end = p.N * (blockIdx.x + 1) / gridDim.x;
    const int nrows = (int)(r_end - r_begin);
    const int nocts = (nrows + MV_ROWS - 1) / MV_ROWS;
    const int my_octs = warp < nocts ? (nocts - 1 - warp) / MV_WARPS + 1 : 0;
    const int nkc = (p.nb + p.kc - 1) / p.kc;
    const int total = my_octs * nkc;  // this warp's stage sequence
    const unsigned FULLM = 0xffffffffu;

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const uint64_t pol = policy_evict_first();
    // issue cursor: next (oct, chunk, stage) to fill; advanced without divisions
    int i_od = 0, i_c = 0, i_s = 0, issued = 0;
    auto issue_next = [&]() {
        const int r0 = (warp + i_od * MV_WARPS) * MV_ROWS;
        const int rq = min(MV_ROWS, nrows - r0);
        const int kl = min(p.kc, p.nb - i_c * p.kc);
        const uint32_t bytes = (uint32_t)kl * Q4K_BYTES;
        if (lane == 0) mbar_arrive_expect_tx(&full[i_s], bytes * (uint32_t)rq);
        __syncwarp();
        if (lane < rq) {
            const uint8_t* src = seg_row(p, r_begin + r0 + lane) + (size_t)i_c * p.kc * Q4K_BYTES;
            bulk_g2s(ring + (size_t)i_s * p.stage_bytes + (size_t)lane * p.row_stride, src, bytes, &full[i_s], pol);
        }
        ++issued;
        if (++i_c == nkc) { i_c = 0; ++i_od; }
        if (++i_s == p.stages) i_s = 0;
    };
    // weights do not depend on the previous kernel: start streaming now
    const int prefill = min(p.stages, total);
    for (int q = 0; q < prefill; ++q) issue_next();
    pdl_trigger();
    pdl_wait();
    stage_activations<FOLD, SRC>(p, act, s_red, threadIdx.x);
    __syncthreads();

    const int rgrp = lane >> 2;  // row of the oct worked by this thread
    const int t = lane & 3;      // owns reference lanes 2t, 2t+1

    float best_v[NB];
    int best_i[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { best_v[b] = -INFINITY; best_i[b] = 0x7fffffff; }

    int consumed = 0, c_s = 0;
    uint32_t c_ph = 0;
    bool ok = true;
    for (int od = 0; od < my_octs && ok; ++od) {
        const int rin = (warp + od * MV_WARPS) * MV_ROWS + rgrp;
        const bool live = rin < nrows;
        float acc0[NB], acc1[NB], accm[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) { acc0[b] = 0.f; acc1[b] = 0.f; accm[b] = 0.f; }

        for (int c = 0; c < nkc; ++c) {
            if (!__all_sync(FULLM, mbar_wait_bounded(&full[c_s], c_ph))) {
                ok = false;
                if (lane == 0) set_status(p.status, ST_TIMEOUT);
                break;
            }
            ++consumed;
            const int kl = min(p.kc, p.nb - c * p.kc);
            // rows past the end of the range read stale (in-bounds) stage bytes
            // and are never stored
            const uint8_t* rowp = ring + (size_t)c_s * p.stage_bytes + (size_t)rgrp * p.row_stride;
            const uint8_t* actc = act + c * p.kc * ACT_BLOCK_BYTES;
#pragma unroll 2
            for (int kb = 0; kb < kl; ++kb) {
                const RowBlk r = decode_row<FOLD>(rowp + kb * Q4K_BYTES, t);
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    fold_block<FOLD, PART>(p, r, actc + (b * p.nb + kb) * ACT_BLOCK_BYTES, t, b, c * p.kc + kb,
                                           r_begin + rin, live, acc0[b], acc1[b], accm[b]);
            }
            __syncwarp();
            if (issued < total) {
                fence_proxy_async_smem();
                issue_next();
            }
            if (++c_s == p.stages) { c_s = 0; c_ph ^= 1u; }
        }
        if (!ok) break;
#pragma unroll
        for (int b = 0; b < NB; ++b)
            finish_row<FOLD, EPI>(p, acc0[b], acc1[b], accm[b], rgrp, t, b, live, r_begin + rin, best_v[b], best_i[b]);
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
                for (int w = 1; w < MV_WARPS; ++w)
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
// Pick kc (super-blocks per row per stage) as large as the shared-memory
// budget allows with at least 4 stages per warp ring (bulk copies of a few
// hundred bytes or more keep the copy engine efficient), capped by the
// per-row copy target.
int matvec_plan(MatvecParams& p, int grid, int smem_cap, int stage_target) {
    if (grid < 1) return BH_EINVAL;
    const int act_bytes = p.B * p.nb * ACT_BLOCK_BYTES;
    const int ring_off = (act_bytes + 127) / 128 * 128;
    int kc = stage_target / Q4K_BYTES;
    if (kc < 1) kc = 1;
    if (kc > p.nb) kc = p.nb;
    for (;; --kc) {
        const int words = kc * (Q4K_BYTES / 4);
        const int padw = ((8 - (words % 32)) % 32 + 32) % 32;  // row stride == 8 words (mod 32 banks)
        const int stride = kc * Q4K_BYTES + 4 * padw;
        const int stage = MV_ROWS * stride;
        int stages = (smem_cap - ring_off - 256) / (MV_WARPS * (stage + 8));
        if (stages > 4) stages = 4;
        if (stages >= 2) {
            p.kc = kc;
            p.row_stride = stride;
            p.stage_bytes = stage;
            p.stages = stages;
            p.rows_per_tile = MV_ROWS;
            p.act_off = 0;
            p.ring_off = ring_off;
            p.bar_off = ring_off + MV_WARPS * stages * stage;
            p.smem_bytes = p.bar_off + MV_WARPS * stages * 8;
            return BH_OK;
        }
        if (kc == 1) return BH_EINVAL;  // activations too large for shared memory
    }
}

template <int FOLD, int NB, int SRC, int EPI, bool PART>
static int launch_t(const MatvecParams& p, const LaunchOpts& o, int grid) {
    auto kern = q4k_matvec_kernel<FOLD, NB, SRC, EPI, PART>;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
            return BH_EIO;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MV_THREADS);
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
    switch (p.B) {
        case 1: return launch_t<FOLD, 1, SRC, EPI, PART>(p, o, grid);
        case 2: return launch_t<FOLD, 2, SRC, EPI, PART>(p, o, grid);
        case 3: return launch_t<FOLD, 3, SRC, EPI, PART>(p, o, grid);
        case 4: return launch_t<FOLD, 4, SRC, EPI, PART>(p, o, grid);
        case 5: return launch_t<FOLD, 5, SRC, EPI, PART>(p, o, grid);
        case 6: return launch_t<FOLD, 6, SRC, EPI, PART>(p, o, grid);
        case 7: return launch_t<FOLD, 7, SRC, EPI, PART>(p, o, grid);
        case 8: return launch_t<FOLD, 8, SRC, EPI, PART>(p, o, grid);
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
    switch (src * 3 + epi) {
        case ACT_Q8K * 3 + EPI_STORE: return launch_nb<FOLD, ACT_Q8K, EPI_STORE, false>(p, o, grid);
        case ACT_Q8K * 3 + EPI_ARGMAX: return launch_nb<FOLD, ACT_Q8K, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32 * 3 + EPI_STORE: return launch_nb<FOLD, ACT_F32, EPI_STORE, false>(p, o, grid);
        case ACT_F32 * 3 + EPI_ADD: return launch_nb<FOLD, ACT_F32, EPI_ADD, false>(p, o, grid);
        case ACT_F32 * 3 + EPI_ARGMAX: return launch_nb<FOLD, ACT_F32, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32_RMSNORM * 3 + EPI_STORE: return launch_nb<FOLD, ACT_F32_RMSNORM, EPI_STORE, false>(p, o, grid);
        case ACT_F32_RMSNORM * 3 + EPI_ARGMAX: return launch_nb<FOLD, ACT_F32_RMSNORM, EPI_ARGMAX, false>(p, o, grid);
        case ACT_F32_SWIGLU * 3 + EPI_ADD: return launch_nb<FOLD, ACT_F32_SWIGLU, EPI_ADD, false>(p, o, grid);
        default: return BH_EINVAL;
    }
}

int launch_matvec(const MatvecParams& p, int fold, int act_src, int epi, const LaunchOpts& o) {
    const int grid = o.grid;
    if (fold == BH_FOLD_X86) return launch_fold<BH_FOLD_X86>(p, act_src, epi, o, grid);
    if (fold == BH_FOLD_GENERIC) return launch_fold<BH_FOLD_GENERIC>(p, act_src, epi, o, grid);
    return BH_EINVAL;
}

}  // namespace bh
