// q8k_device.cuh — warp-level Q8_K quantization of one 256-value block and
// the staged (lane-permuted) activation layout the matvec consumes.
#pragma once

#include "bh_common.cuh"

namespace bh {

// One warp quantizes one block of 256 floats; lane l owns values 8l..8l+7.
// Restates quantize_row_q8_K_ref (ggml-quants.c:2692-2729):
//   vmax  = the value of largest |x| (first such index on ties),
//   iscale = -127 / vmax, q = min(127, round_half_even(iscale * x)),
//   d = 1 / iscale, bsums[g] = sum of q over 16 values; all-zero -> d = 0.
// Every operation is a correctly rounded binary32 operation, as on the CPU
// when compiled without FMA contraction.
struct Q8Block {
    int q[8];      // this lane's eight codes
    float d;       // block scale (same on every lane)
    int bsum16;    // sum of the lane pair's 16 codes (valid on every lane)
};

__device__ __forceinline__ Q8Block q8k_quantize_warp(const float (&v)[8], int lane) {
    // local first-max of |x| over increasing positions
    float best = 0.f, bval = 0.f;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const float a = fabsf(v[t]);
        if (a > best) { best = a; bval = v[t]; bidx = 8 * lane + t; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const float ov = __shfl_xor_sync(0xffffffffu, bval, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, off);
        if (ob > best || (ob == best && oi < bidx)) { best = ob; bval = ov; bidx = oi; }
    }
    Q8Block r;
    if (best == 0.f) {
#pragma unroll
        for (int t = 0; t < 8; ++t) r.q[t] = 0;
        r.d = 0.f;
        r.bsum16 = 0;
        return r;
    }
    const float iscale = __fdiv_rn(-127.f, bval);
    int s = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int c = round_biased(__fmul_rn(iscale, v[t]));
        r.q[t] = c < 127 ? c : 127;
        s += r.q[t];
    }
    r.bsum16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    r.d = __fdiv_rn(1.f, iscale);
    return r;
}

// Staged activation block (ACT_BLOCK_BYTES = 304):
//   bytes   0..271 : q8 codes as 64 words, lane-major: lane m's 8 words (32
//                    bytes) at act_lane_off(m) = 32 m, plus 16 for m >= 4, so
//                    the 16-byte reads of the lanes a warp reads together fall
//                    on distinct banks (without the gap lanes m and m + 4 sit
//                    128 bytes apart, on the same banks)
//   bytes 272..275 : d (float)
//   bytes 288..303 : S[t] = bsums[2t] + bsums[2t+1], t = 0..7, as int16;
//                    word k = (S[2k], S[2k+1]) feeds one dp2a with two 6-bit mins
// Word slot layout per fold (lane = the 8-way split of a row's work):
//   FOLD_X86 (lane m):     slot 2j   = codes 64j + 4m .. +3       (low-nibble half)
//                          slot 2j+1 = codes 64j + 32 + 4m .. +3  (high-nibble half)
//   FOLD_GENERIC (lane l): slot 2g   = codes 64g + l + 8c, c = 0..3
//                          slot 2g+1 = codes 64g + 32 + l + 8c, c = 0..3
// i.e. each staged word holds exactly the four codes one dp4a of that lane needs.
template <int FOLD>
__device__ __forceinline__ int staged_byte_offset(int p) {
    if (FOLD == BH_FOLD_X86) {
        const int g = p >> 6, h = (p >> 5) & 1, m = (p & 31) >> 2;
        return act_lane_off(m) + (2 * g + h) * 4 + (p & 3);
    } else {
        const int g = p >> 6, h = (p >> 5) & 1, r = p & 31;
        const int l = r & 7, c = r >> 3;
        return act_lane_off(l) + (2 * g + h) * 4 + c;
    }
}

// Write this lane's 8 codes (positions 8*lane .. +7) into a staged block.
template <int FOLD>
__device__ __forceinline__ void stage_codes(uint8_t* blk, const int (&q)[8], int lane) {
    if (FOLD == BH_FOLD_X86) {
        // positions 8l..8l+3 and 8l+4..8l+7 are whole staged words
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int p = 8 * lane + 4 * h;
            const uint32_t w = (uint32_t)(q[4 * h] & 0xff) | ((uint32_t)(q[4 * h + 1] & 0xff) << 8) |
                               ((uint32_t)(q[4 * h + 2] & 0xff) << 16) | ((uint32_t)(q[4 * h + 3] & 0xff) << 24);
            *reinterpret_cast<uint32_t*>(blk + staged_byte_offset<FOLD>(p)) = w;
        }
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) blk[staged_byte_offset<FOLD>(8 * lane + t)] = (uint8_t)(q[t] & 0xff);
    }
}

// Write the block scalars: d from lane 0, S[t] from lane 4t (bsum16 is the
// sum over lanes 2g, 2g+1; S[t] = bsum16(lane 4t) + bsum16(lane 4t+2)).
__device__ __forceinline__ void stage_scalars(uint8_t* blk, float d, int bsum16, int lane) {
    const int pair = bsum16 + __shfl_xor_sync(0xffffffffu, bsum16, 2);
    if (lane == 0) *reinterpret_cast<float*>(blk + ACT_D_OFF) = d;
    if ((lane & 3) == 0) reinterpret_cast<int16_t*>(blk + ACT_S_OFF)[lane >> 2] = (int16_t)pair;
}

}  // namespace bh
