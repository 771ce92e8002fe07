// bh_math.cuh — the exponential and SiLU of the decode glue (SwiGLU of the
// dense FFN and of the routed experts, softmax of the router logits),
// evaluated exactly as the reference's x86 CPU backend evaluates them, so
// the device and the reference agree bit for bit.
//
// exp_ggml is one lane of ggml's AVX2 ggml_v_expf (ggml-cpu/vec.h:1233-1271),
// itself the method of ARM's optimized-routines expf: n = round(x / ln2)
// through the 1.5*2^23 shift, the reduced argument b = x - n*ln2 in two
// fused steps (ln2 split in a high and a low part), a degree-5 polynomial
// j ~ exp(b) - 1 in Estrin form, k = 2^n assembled in the exponent field,
// and exp = k + k*j; for |n| > 126 the scale is applied as two factors
// (s2 * s1) so a subnormal or overflowing result rounds once, and |n| > 192
// saturates to s1*s1 (0 or inf). Every step is a single correctly rounded
// binary32 operation (the intrinsics the reference uses are too), written
// with the __f*_rn intrinsics so no contraction or reassociation can change
// it. The oracle (oracle/q4k_oracle.c bho_expf) restates the same sequence
// in C, and both are checked against the reference's compiled vec.cpp.
//
// The reference evaluates the n % 8 tail of a soft_max row or a SiLU row
// with libm expf instead; every length on this path (128 experts, n_ff
// multiples of 256) has no tail.
#pragma once

#include "bh_common.cuh"

namespace bh {

__device__ __forceinline__ float exp_ggml(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float n = __fsub_rn(z, r);
    const float b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, __fmaf_rn(-n, 0x1.62e4p-1f, x));
    const uint32_t e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + 0x3f800000u);
    const float u = __fmul_rn(b, b);
    const float j = __fmaf_rn(__fmaf_rn(__fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                                        __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                              u, __fmul_rn(0x1.ffffecp-1f, b));
    if (!(fabsf(n) > 126.f)) return __fmaf_rn(j, k, k);
    const uint32_t g = n <= 0.f ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(g + 0x7f000000u);
    const float s2 = __uint_as_float(e - g);
    if (fabsf(n) > 192.f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}

// silu(x) = x / (1 + exp(0 - x)), one lane of ggml_v_silu (ggml-cpu/vec.h:
// 1273-1280) as ggml_vec_silu_f32 (vec.cpp:396) applies it.
__device__ __forceinline__ float silu_ggml(float x) {
    return __fdiv_rn(x, __fadd_rn(1.f, exp_ggml(__fsub_rn(0.f, x))));
}

// sum / n in double, as rms_norm_f32's mean: when n is a power of two the
// quotient is an exact scaling, so a multiply by 2^-log2(n) gives the same
// bits without the division's latency.
__device__ __forceinline__ double div_by_count(double sum, int n) {
    if ((n & (n - 1)) == 0) {
        const int sh = __ffs(n) - 1;
        return __dmul_rn(sum, __longlong_as_double((long long)(1023 - sh) << 52));
    }
    return __ddiv_rn(sum, (double)n);
}

}  // namespace bh
