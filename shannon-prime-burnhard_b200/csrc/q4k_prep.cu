// q4k_prep.cu — Q8_K activation quantizer, Q4_K weight quantizer (weight
// prep), Q4_K dequantizer and the argmax finisher, all for sm_100a.
//
// The quantizers are bit-exact restatements of the reference's C code
// evaluated with every float operation separately rounded (written with the
// __f*_rn intrinsics, so no contraction can change them).
#include "bh_common.cuh"
#include "bh_kernels.cuh"
#include "q8k_device.cuh"

namespace bh {

// ---------------------------------------------------------------------------
// Q8_K: one warp per 256-value block, GGML block_q8_K output
// (ggml-quants.c:2692-2729 via q8k_quantize_warp).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) q8k_quantize_kernel(const float* __restrict__ x, int64_t nblk,
                                                           uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t blk = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (blk >= nblk) return;
    const float* src = x + blk * QK + 8 * lane;
    const float4 a0 = *reinterpret_cast<const float4*>(src), a1 = *reinterpret_cast<const float4*>(src + 4);
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const Q8Block qb = q8k_quantize_warp(v, lane);
    uint8_t* dst = out + blk * Q8K_BYTES;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        w0 |= (uint32_t)(qb.q[t] & 0xff) << (8 * t);
        w1 |= (uint32_t)(qb.q[4 + t] & 0xff) << (8 * t);
    }
    reinterpret_cast<uint32_t*>(dst + 4)[2 * lane] = w0;
    reinterpret_cast<uint32_t*>(dst + 4)[2 * lane + 1] = w1;
    if (lane == 0) *reinterpret_cast<float*>(dst) = qb.d;
    if ((lane & 1) == 0) reinterpret_cast<int16_t*>(dst + 260)[lane >> 1] = (int16_t)qb.bsum16;
}

int launch_q8k_quantize(const float* x, int64_t K, int B, uint8_t* out, int*, cudaStream_t s) {
    const int64_t nblk = (int64_t)B * (K / QK);
    if (nblk == 0) return BH_OK;
    const int64_t grid = (nblk + 7) / 8;
    q8k_quantize_kernel<<<(unsigned)grid, 256, 0, s>>>(x, nblk, out);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

// ---------------------------------------------------------------------------
// Q4_K weight quantizer: 8 threads per super-block, one per 32-value
// sub-block. quantize_row_q4_K_ref (ggml-quants.c:1395-1465) with
// make_qkx2_quants (ggml-quants.c:737-816: nmax 15, rmin -1, rdelta 0.1,
// nstep 20, squared error, weights sqrt(mean(x^2)) + |x|).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ float fit_subblock(const float (&x)[32], const float (&w)[32], uint8_t (&L)[32], float* neg_min) {
    float lo = x[0], hi = x[0];
    float sw = w[0];
    float sx = __fmul_rn(sw, x[0]);
#pragma unroll
    for (int i = 1; i < 32; ++i) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
        sw = __fadd_rn(sw, w[i]);
        sx = __fadd_rn(sx, __fmul_rn(w[i], x[i]));
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
#pragma unroll
        for (int i = 0; i < 32; ++i) L[i] = 0;
        *neg_min = -lo;
        return 0.f;
    }
    // the range is re-derived from the current min on every use: the search
    // below may move min, and later trial scales are taken over hi - min
    float inv = __fdiv_rn(15.f, __fsub_rn(hi, lo));
    float scale = __fdiv_rn(1.f, inv);
    float best = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int l = clampi(round_biased(__fmul_rn(inv, __fsub_rn(x[i], lo))), 0, 15);
        L[i] = (uint8_t)l;
        float diff = __fsub_rn(__fadd_rn(__fmul_rn(scale, (float)l), lo), x[i]);
        diff = __fmul_rn(diff, diff);
        best = __fadd_rn(best, __fmul_rn(w[i], diff));
    }
    for (int is = 0; is <= 20; ++is) {
        inv = __fdiv_rn(__fadd_rn(__fadd_rn(-1.f, __fmul_rn(0.1f, (float)is)), 15.f), __fsub_rn(hi, lo));
        float s_l = 0.f, s_l2 = 0.f, s_xl = 0.f;
        uint8_t trial[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int l = clampi(round_biased(__fmul_rn(inv, __fsub_rn(x[i], lo))), 0, 15);
            trial[i] = (uint8_t)l;
            const float wl = __fmul_rn(w[i], (float)l);
            s_l = __fadd_rn(s_l, wl);
            s_l2 = __fadd_rn(s_l2, __fmul_rn(wl, (float)l));
            s_xl = __fadd_rn(s_xl, __fmul_rn(wl, x[i]));
        }
        const float D = __fsub_rn(__fmul_rn(sw, s_l2), __fmul_rn(s_l, s_l));
        if (D > 0) {
            float t_scale = __fdiv_rn(__fsub_rn(__fmul_rn(sw, s_xl), __fmul_rn(sx, s_l)), D);
            float t_min = __fdiv_rn(__fsub_rn(__fmul_rn(s_l2, sx), __fmul_rn(s_l, s_xl)), D);
            if (t_min > 0) {
                t_min = 0;
                t_scale = __fdiv_rn(s_xl, s_l2);
            }
            float err = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float diff = __fsub_rn(__fadd_rn(__fmul_rn(t_scale, (float)trial[i]), t_min), x[i]);
                diff = __fmul_rn(diff, diff);
                err = __fadd_rn(err, __fmul_rn(w[i], diff));
            }
            if (err < best) {
#pragma unroll
                for (int i = 0; i < 32; ++i) L[i] = trial[i];
                best = err;
                scale = t_scale;
                lo = t_min;
            }
        }
    }
    *neg_min = -lo;
    return scale;
}

__global__ void __launch_bounds__(256) q4k_quantize_kernel(const float* __restrict__ src, int64_t nsb,
                                                           uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int j = lane & 7;  // sub-block of this thread
    const int64_t sb = (int64_t)blockIdx.x * 32 + (threadIdx.x >> 3);
    const bool live = sb < nsb;
    const unsigned FULLM = 0xffffffffu;

    float x[32], w[32];
    uint8_t L[32];
    float scale = 0.f, nmin = 0.f;
    if (live) {
        const float* xs = src + sb * QK + 32 * j;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float4 v = reinterpret_cast<const float4*>(xs)[t];
            x[4 * t] = v.x; x[4 * t + 1] = v.y; x[4 * t + 2] = v.z; x[4 * t + 3] = v.w;
        }
        float ss = 0.f;
#pragma unroll
        for (int t = 0; t < 32; ++t) ss = __fadd_rn(ss, __fmul_rn(x[t], x[t]));
        const float av = __fsqrt_rn(__fdiv_rn(ss, 32.f));
#pragma unroll
        for (int t = 0; t < 32; ++t) w[t] = __fadd_rn(av, fabsf(x[t]));
        scale = fit_subblock(x, w, L, &nmin);
    }
    // super-block maxima over the 8 sub-blocks (max is order independent)
    float max_scale = scale > 0.f ? scale : 0.f, max_min = nmin > 0.f ? nmin : 0.f;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) {
        const float os = __shfl_xor_sync(FULLM, max_scale, off);
        const float om = __shfl_xor_sync(FULLM, max_min, off);
        if (os > max_scale) max_scale = os;
        if (om > max_min) max_min = om;
    }
    const float inv_scale = max_scale > 0 ? __fdiv_rn(63.f, max_scale) : 0.f;
    const float inv_min = max_min > 0 ? __fdiv_rn(63.f, max_min) : 0.f;
    int ls = (uint8_t)round_biased(__fmul_rn(inv_scale, scale));
    int lm = (uint8_t)round_biased(__fmul_rn(inv_min, nmin));
    ls = ls > 63 ? 63 : ls;
    lm = lm > 63 ? 63 : lm;
    const int ls_hi = __shfl_down_sync(FULLM, ls, 4);  // from sub-block j+4
    const int lm_hi = __shfl_down_sync(FULLM, lm, 4);
    // packed bytes: j<4: scales[j] = ls_j | (ls_{j+4} >> 4) << 6, scales[j+4] = lm_j | (lm_{j+4} >> 4) << 6;
    //               j>=4: scales[j+4] = (ls_j & 15) | (lm_j & 15) << 4
    const uint16_t hd = __half_as_ushort(__float2half_rn(__fdiv_rn(max_scale, 63.f)));
    const uint16_t hm = __half_as_ushort(__float2half_rn(__fdiv_rn(max_min, 63.f)));
    uint8_t sc6 = 0, mn6 = 0;  // this sub-block's 6-bit scale / min as stored
    sc6 = (uint8_t)ls;
    mn6 = (uint8_t)lm;
    uint8_t* blk = out + sb * Q4K_BYTES;
    if (live) {
        if (j < 4) {
            blk[4 + j] = (uint8_t)(ls | ((ls_hi >> 4) << 6));
            blk[8 + j] = (uint8_t)(lm | ((lm_hi >> 4) << 6));
        } else {
            blk[8 + j] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
        }
        if (j == 0) {
            reinterpret_cast<uint16_t*>(blk)[0] = hd;
            reinterpret_cast<uint16_t*>(blk)[1] = hm;
        }
        // second pass with the rounded super-block scales
        const float d = __fmul_rn(h2f(hd), (float)sc6);
        if (d != 0.f) {
            const float dm = __fmul_rn(h2f(hm), (float)mn6);
#pragma unroll
            for (int t = 0; t < 32; ++t) L[t] = (uint8_t)clampi(round_biased(__fdiv_rn(__fadd_rn(x[t], dm), d)), 0, 15);
        }
    }
    // qs[32g + t] = L_{2g}[t] | L_{2g+1}[t] << 4: even threads gather odd neighbours' codes
    uint32_t packed[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
        packed[k] = (uint32_t)L[4 * k] | ((uint32_t)L[4 * k + 1] << 8) | ((uint32_t)L[4 * k + 2] << 16) |
                    ((uint32_t)L[4 * k + 3] << 24);
    uint32_t hiw[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) hiw[k] = __shfl_down_sync(FULLM, packed[k], 1);
    if (live && (j & 1) == 0) {
        uint32_t* qs = reinterpret_cast<uint32_t*>(blk + 16 + 32 * (j >> 1));
#pragma unroll
        for (int k = 0; k < 8; ++k) qs[k] = packed[k] | (hiw[k] << 4);
    }
}

int launch_q4k_quantize(const float* w, int64_t N, int64_t K, uint8_t* out, cudaStream_t s) {
    const int64_t nsb = N * (K / QK);
    if (nsb == 0) return BH_OK;
    q4k_quantize_kernel<<<(unsigned)((nsb + 31) / 32), 256, 0, s>>>(w, nsb, out);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

// ---------------------------------------------------------------------------
// Q4_K -> fp32 (dequantize_row_q4_K, ggml-quants.c:1467-1489): one thread
// per 8 outputs.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) q4k_dequantize_kernel(const uint8_t* __restrict__ w, int64_t nsb,
                                                             float* __restrict__ out) {
    const int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x;
    const int64_t sb = t >> 5;
    if (sb >= nsb) return;
    const int part = (int)(t & 31);          // 8 consecutive outputs: positions 8*part..
    const uint8_t* blk = w + sb * Q4K_BYTES;
    const float d = h2f(reinterpret_cast<const uint16_t*>(blk)[0]);
    const float dmin = h2f(reinterpret_cast<const uint16_t*>(blk)[1]);
    const int p0 = 8 * part;
    const int j = p0 >> 5, g = p0 >> 6, hi = (p0 >> 5) & 1;
    const uint8_t* q = blk + 4;
    int sc, mn;
    if (j < 4) { sc = q[j] & 63; mn = q[j + 4] & 63; }
    else { sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    const uint8_t* qs = blk + 16 + 32 * g + (p0 & 31);
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int c = hi ? (qs[k] >> 4) : (qs[k] & 0xF);
        o[k] = __fsub_rn(__fmul_rn(d1, (float)c), m1);
    }
    float4* dst = reinterpret_cast<float4*>(out + sb * QK + p0);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
}

int launch_q4k_dequantize(const uint8_t* w, int64_t N, int64_t K, float* out, cudaStream_t s) {
    const int64_t nsb = N * (K / QK);
    if (nsb == 0) return BH_OK;
    q4k_dequantize_kernel<<<(unsigned)((nsb * 32 + 255) / 256), 256, 0, s>>>(w, nsb, out);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

// ---------------------------------------------------------------------------
// argmax finisher: reduce per-CTA (max, first index) candidates per column.
// Same result as engine.cpp:36-43 (strict >, first maximum wins) because
// candidates carry the smallest index among equal maxima.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) argmax_finish_kernel(const float* __restrict__ cv, const int32_t* __restrict__ ci,
                                                            int ncand, int B, int32_t* tok, float* val,
                                                            const int* status) {
    pdl_wait();
    // a bounded wait of the matvec before it ran out (status set): no token
    const bool failed = status && *reinterpret_cast<const volatile int*>(status) != ST_OK;
    __shared__ float sv[8];
    __shared__ int si[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = 0; b < B; ++b) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = threadIdx.x; c < ncand; c += blockDim.x) {
            const float v = cv[c * B + b];
            const int i = ci[c * B + b];
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
            if (bi == 0x7fffffff) bi = 0;  // all candidates NaN: index 0, as the CPU loop leaves it
            tok[b] = failed ? -1 : bi;
            if (val) val[b] = bv;
        }
        __syncthreads();
    }
}

int launch_argmax_finish(const float* cand_val, const int32_t* cand_idx, int ncand, int B, int32_t* tok_out,
                         float* val_out, cudaStream_t s, bool pdl, const int* status) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    static std::atomic<uint64_t> attr_devices{0};
    // the same shared-memory carveout as the matvec it follows (no SM reconfiguration between them)
    if (!attrs_on_device(attr_devices, [] {
            return cudaFuncSetAttribute(argmax_finish_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared) == cudaSuccess;
        }))
        return BH_EIO;
    return cudaLaunchKernelEx(&cfg, argmax_finish_kernel, cand_val, cand_idx, ncand, B, tok_out, val_out, status) ==
                   cudaSuccess
               ? BH_OK
               : BH_EIO;
}

}  // namespace bh
