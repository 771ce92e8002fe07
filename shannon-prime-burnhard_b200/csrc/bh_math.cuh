// bh_math.cuh — the exponential used by the routed-expert glue (softmax of
// the router logits, SiLU of the gate), written so that the CPU oracle can
// evaluate the identical sequence of correctly rounded binary32 operations
// and the GPU results match it bit for bit.
//
// Method: Cody–Waite argument reduction (W. J. Cody and W. Waite, "Software
// Manual for the Elementary Functions", 1980): x = n*ln2 + r with
// n = round(x * log2(e)) and ln2 split into a 15-bit-exact high part and a
// low part, |r| <= ~0.35; then exp(r) from its Taylor series to degree 7
// (coefficients 1/k!, each rounded to binary32) in Horner form with fused
// multiply-adds; then the scale 2^n applied as two exact powers of two so a
// subnormal result is rounded once. The truncation error is below 0.13 ulp
// and the evaluated error stays within 1 ulp of exp(x) (checked on the CPU
// against a double-precision exp over the float range the callers use).
//
// The reference evaluates these with ggml's SIMD exponential
// (ggml-cpu/vec.h, ggml_v_expf) or libm expf; results agree with it to a few
// ulp, which is within the fp32 tolerance of the path.
#pragma once

#include "bh_common.cuh"

namespace bh {

__device__ __forceinline__ float exp_cw(float x) {
    if (!(x == x)) return x;                                    // NaN
    if (x > 0x1.62e430p+6f) return __int_as_float(0x7f800000);  // above ln(FLT_MAX): +inf
    if (x < -103.972084f) return 0.f;                           // below ln(2^-150): rounds to zero
    const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));        // round(x / ln2), ties to even
    float r = __fmaf_rn(-n, 0x1.62e400p-1f, x);                 // ln2 high part (n * hi is exact)
    r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);                      // ln2 low part
    float q = 0x1.a01a02p-13f;                                  // 1/7!
    q = __fmaf_rn(q, r, 0x1.6c16c2p-10f);                       // 1/6!
    q = __fmaf_rn(q, r, 0x1.111112p-7f);                        // 1/5!
    q = __fmaf_rn(q, r, 0x1.555556p-5f);                        // 1/4!
    q = __fmaf_rn(q, r, 0x1.555556p-3f);                        // 1/3!
    q = __fmaf_rn(q, r, 0.5f);
    q = __fmaf_rn(q, r, 1.f);
    q = __fmaf_rn(q, r, 1.f);
    const int ni = (int)n;                                      // -150 .. 128
    const int n1 = ni >> 1, n2 = ni - n1;                       // both within [-75, 64]
    return __fmul_rn(__fmul_rn(q, __int_as_float((n1 + 127) << 23)), __int_as_float((n2 + 127) << 23));
}

// silu(x) = x / (1 + exp(-x))   (ggml_silu_f32, ggml-cpu/vec.h:1064)
__device__ __forceinline__ float silu_cw(float x) { return __fdiv_rn(x, __fadd_rn(1.f, exp_cw(-x))); }

}  // namespace bh
