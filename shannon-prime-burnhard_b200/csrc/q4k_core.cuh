// q4k_core.cuh — the per-super-block arithmetic shared by the dense and the
// routed-expert matvec kernels: decode of one block_q4_K for one thread,
// the exact integer lane sums, and the reference's fp32 fold.
//
// TPR threads work one row (TPR = 4: thread t owns reference lanes 2t, 2t+1;
// TPR = 8: thread t owns lane t; TPR = 16, x86 fold only: threads t and t ^ 8
// share lane t & 7, each taking two of the four 32-byte quant groups, and add
// their integer halves before the fold). Integer sums are exact (|partial| <
// 2^24), so only the fp32 order matters, and it is reproduced operation by
// operation:
//   FOLD_X86     (ggml-cpu/arch/x86/quants.c:1900-1983): lane m = bytes
//                4m..4m+3 of every 32-byte quant group; acc = fma(d, sumi, acc).
//   FOLD_GENERIC (ggml-cpu/quants.c:645-718): lane l = positions p % 8 == l;
//                sums += d * aux, sumf -= dmin * sumi, then sumf += sums[0..7].
#pragma once

#include "bh_common.cuh"

namespace bh {

// ---------------------------------------------------------------------------
// per-super-block work of one thread
// ---------------------------------------------------------------------------
// TPR threads work one row (TPR = 4: thread t owns reference lanes 2t, 2t+1;
// TPR = 8: thread t owns lane t; TPR = 16: thread t owns half t >> 3 of lane
// t & 7); every thread also computes min lane t & 3 (the threads above 3
// repeat 0..3 and are not summed).
template <int TPR>
struct RowBlk {
    static constexpr int L = TPR >= 8 ? 1 : 8 / TPR;  // reference lanes per thread
    static constexpr int G = TPR == 16 ? 2 : 4;       // 32-byte quant groups per thread
    float fd, fdm;
    uint32_t sc03, sc47, mnk;          // mnk: the two mins of min lane t & 3 in bytes 0..1
    uint32_t lo[L][G], hi[L][G];       // (TPR = 16: sc03 holds the scales of this thread's groups)
};

template <int FOLD, int TPR>
__device__ __forceinline__ RowBlk<TPR> decode_row(const uint8_t* blk, int t) {
    constexpr int L = RowBlk<TPR>::L;
    RowBlk<TPR> r;
    const uint4 h = *reinterpret_cast<const uint4*>(blk);
    r.fd = h2f((uint16_t)(h.x & 0xffffu));
    r.fdm = h2f((uint16_t)(h.x >> 16));
    // 6-bit scales/mins, get_scale_min_k4 (ggml-quants.c:818-825) word-wise:
    // j<4: sc = q[j] & 63, mn = q[j+4] & 63;
    // j>=4: sc = (q[j+4] & 15) | (q[j-4] >> 6) << 4, mn = (q[j+4] >> 4) | (q[j] >> 6) << 4
    r.sc03 = h.y & 0x3f3f3f3fu;
    r.sc47 = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const int k = t & 3;
    const uint32_t mn = (k & 2) ? (((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3f3f3f3fu);
    r.mnk = mn >> ((k & 1) * 16);
    const uint32_t* qs = reinterpret_cast<const uint32_t*>(blk + 16);
    static_assert(TPR != 16 || FOLD == BH_FOLD_X86, "16 threads per row: x86 fold only");
    if (TPR == 16) {
        // groups 2h, 2h + 1 (sub-blocks 4h .. 4h + 3) of lane t & 7, h = t >> 3
        const int h2 = t >> 3, m = t & 7;
        if (h2) r.sc03 = r.sc47;
#pragma unroll
        for (int g = 0; g < RowBlk<TPR>::G; ++g) {
            const uint32_t w = qs[8 * (2 * h2 + g) + m];
            r.lo[0][g] = w & 0x0f0f0f0fu;
            r.hi[0][g] = (w >> 4) & 0x0f0f0f0fu;
        }
    } else if (FOLD == BH_FOLD_X86) {
        // lane m = bytes 4m..4m+3 of each 32-byte group: word m
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint32_t w[L];
            if (L == 2) {
                const uint2 w2 = *reinterpret_cast<const uint2*>(qs + 8 * g + 2 * t);
                w[0] = w2.x;
                w[L - 1] = w2.y;
            } else {
                w[0] = qs[8 * g + t];
            }
#pragma unroll
            for (int e = 0; e < L; ++e) {
                r.lo[e][g] = w[e] & 0x0f0f0f0fu;
                r.hi[e][g] = (w[e] >> 4) & 0x0f0f0f0fu;
            }
        }
    } else {
        // lane l = group bytes l, l+8, l+16, l+24: a byte gather from words
        // l/4 + {0,2,4,6} (the lanes of one thread share those words)
        const int l0 = t * L, k0 = l0 >> 2, tb = l0 & 3;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint32_t* gw = qs + 8 * g;
            const uint32_t w0 = gw[k0], w1 = gw[k0 + 2], w2 = gw[k0 + 4], w3 = gw[k0 + 6];
#pragma unroll
            for (int e = 0; e < L; ++e) {
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

// Half a lane's sum (two quant groups = four sub-blocks, their scales in the
// bytes of sc): the TPR = 16 split.
__device__ __forceinline__ int lane_sum_half(const uint32_t (&lo)[2], const uint32_t (&hi)[2], uint32_t sc,
                                             const int4 a) {
    const int d0 = dp4a((int)lo[0], a.x, 0), d1 = dp4a((int)hi[0], a.y, 0);
    const int d2 = dp4a((int)lo[1], a.z, 0), d3 = dp4a((int)hi[1], a.w, 0);
    const int s = __dp2a_lo((int)__byte_perm((uint32_t)d0, (uint32_t)d1, 0x5410), (int)sc, 0);
    return __dp2a_hi((int)__byte_perm((uint32_t)d2, (uint32_t)d3, 0x5410), (int)sc, s);
}

// Sum over the 4 min lanes held by threads t & 3 = 0..3 of a row (exact ints).
template <int TPR>
__device__ __forceinline__ int sum_min_lanes(int v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// One activation column applied to one decoded row block: the reference's
// per-block fp32 step for this thread's lanes and its min lane. With PART,
// the row's exact sub-block sums and min term are also reduced and, when
// part_dst is non-null, written by thread 0 as 9 int32.
template <int FOLD, bool PART, int TPR>
__device__ __forceinline__ void fold_block(const RowBlk<TPR>& r, const uint8_t* A, int t, int32_t* part_dst,
                                           float (&acc)[RowBlk<TPR>::L], float& accm) {
    constexpr int L = RowBlk<TPR>::L;
    static_assert(TPR != 16 || !PART, "16 threads per row: no partials");
    const float yd = *reinterpret_cast<const float*>(A + ACT_D_OFF);
    const int spk = reinterpret_cast<const int*>(A + ACT_S_OFF)[t & 3];
    int li[L];
    int sub[L][8];
    if constexpr (TPR == 16) {
        // this thread's half of lane t & 7, then the other half from thread t ^ 8
        const int4 a = *reinterpret_cast<const int4*>(A + act_lane_off(t & 7) + 16 * (t >> 3));
        const int hs = lane_sum_half(r.lo[0], r.hi[0], r.sc03, a);
        li[0] = hs + __shfl_xor_sync(0xffffffffu, hs, 8);
    } else {
#pragma unroll
        for (int e = 0; e < L; ++e) {
            const int4 a0 = *reinterpret_cast<const int4*>(A + act_lane_off(t * L + e));
            const int4 a1 = *reinterpret_cast<const int4*>(A + act_lane_off(t * L + e) + 16);
            li[e] = lane_sum(r.lo[e], r.hi[e], r.sc03, r.sc47, a0, a1, sub[e], PART);
        }
    }
    const int mp = __dp2a_lo(spk, (int)r.mnk, 0);
    if (FOLD == BH_FOLD_X86) {
        // acc[m] = fma(y.d * fp16(d), sumi[m], acc[m]);
        // accm[k] = fma(-y.d * fp16(dmin), min_{2k} S_{2k} + min_{2k+1} S_{2k+1}, accm[k])
        const float d = __fmul_rn(yd, r.fd);
#pragma unroll
        for (int e = 0; e < L; ++e) acc[e] = __fmaf_rn(d, i2f_exact(li[e]), acc[e]);
        accm = __fmaf_rn(__fmul_rn(-yd, r.fdm), i2f_exact(mp), accm);
    } else {
        // sums[l] += (fp16(d) * y.d) * aux[l];  sumf -= (fp16(dmin) * y.d) * sumi
        const float d = __fmul_rn(r.fd, yd);
#pragma unroll
        for (int e = 0; e < L; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(d, i2f_exact(li[e])));
        const int sumi = sum_min_lanes<TPR>(mp);
        accm = __fsub_rn(accm, __fmul_rn(__fmul_rn(r.fdm, yd), i2f_exact(sumi)));
    }
    if (PART) {
        const int msum = sum_min_lanes<TPR>(mp);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int v = 0;
#pragma unroll
            for (int e = 0; e < L; ++e) v += sub[e][j];
#pragma unroll
            for (int off = 1; off < TPR; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            sub[0][j] = v;
        }
        if (part_dst && t == 0) {
            for (int j = 0; j < 8; ++j) part_dst[j] = sub[0][j];
            part_dst[8] = msum;
        }
    }
}

// The row's dot product from its threads' lane accumulators, combined in the
// reference's order; every thread of the row returns the same value.
template <int FOLD, int TPR>
__device__ __forceinline__ float row_value(const float (&acc)[RowBlk<TPR>::L], float accm, int rgrp) {
    const unsigned FULLM = 0xffffffffu;
    if (FOLD == BH_FOLD_X86) {
        // hsum_float_8 (arch/x86/quants.c:43-49): ((a4+a0)+(a6+a2)) + ((a5+a1)+(a7+a3))
        float hs;
        if (TPR == 4) {
            // thread t holds lanes 2t (acc[0]) and 2t+1 (acc[1])
            const float x0 = __fadd_rn(acc[0], __shfl_xor_sync(FULLM, acc[0], 2));  // t0: a0+a4, t1: a2+a6
            const float x1 = __fadd_rn(acc[RowBlk<TPR>::L - 1], __shfl_xor_sync(FULLM, acc[RowBlk<TPR>::L - 1], 2));
            const float y0 = __fadd_rn(x0, __shfl_xor_sync(FULLM, x0, 1));
            const float y1 = __fadd_rn(x1, __shfl_xor_sync(FULLM, x1, 1));
            hs = __fadd_rn(y0, y1);
        } else {
            // thread t holds lane t & 7 (TPR = 16: both halves hold it)
            const float t1 = __fadd_rn(acc[0], __shfl_xor_sync(FULLM, acc[0], 4));  // t0: a0+a4
            const float t2 = __fadd_rn(t1, __shfl_xor_sync(FULLM, t1, 2));          // t0: (a0+a4)+(a2+a6)
            hs = __fadd_rn(t2, __shfl_xor_sync(FULLM, t2, 1));
        }
        // 4-lane min accumulator, lane k in thread k: (m0+m2) + (m1+m3)
        const float u = __fadd_rn(accm, __shfl_xor_sync(FULLM, accm, 2));
        const float hm = __fadd_rn(u, __shfl_xor_sync(FULLM, u, 1));
        return __fadd_rn(hs, hm);
    } else {
        // sumf (the min chain) += sums[0..7] in order
        constexpr int L = RowBlk<TPR>::L;
        float v = accm;
#pragma unroll
        for (int l = 0; l < 8; ++l) v = __fadd_rn(v, __shfl_sync(FULLM, acc[l % L], rgrp * TPR + l / L));
        return v;
    }
}

}  // namespace bh
