// q6k_matvec.cu — the Q6_K x Q8_K matvec (batch 1..8) on sm_100a.
//
// Real Q4_K_M model files carry some matrices in Q6_K (block_q6_K,
// ggml-common.h:352-357: ql[128] low 4 bits, qh[64] high 2 bits, scales[16]
// int8, fp16 d; 210 bytes per 256 values), which the reference multiplies with
// the same Q8_K activations through ggml_vec_dot_q6_K_q8_K. This kernel
// reproduces the x86 AVX2 branch of that function
// (ggml-cpu/arch/x86/quants.c:2288-2370) bit for bit:
//  - lane m (0..7) of the int32 accumulator takes bytes 4m..4m+3 of each of
//    the 8 vectors of 32 codes (vector is = 4 j + x of half j), each byte the
//    6-bit code q = low nibble (x < 2) or high nibble of ql[64 j + 32 (x & 1)
//    + b] with bits 2x..2x+1 of qh[32 j + b] above it, against q8[128 j + 32 x
//    + b]; the vector's products are scaled by scales[2 is] (m < 4) or
//    scales[2 is + 1] (m >= 4);
//  - minus 32 * (bsums[2m] scales[2m] + bsums[2m+1] scales[2m+1]) (the codes'
//    offset of 32);
//  - acc[m] = fma(y.d * fp16(d), (float)sumi[m], acc[m]) per block, in block
//    order; the row value is hsum_float_8 of the 8 lanes.
// Thread m of a row holds lane m. The 210-byte blocks are only 2-byte
// aligned, so a 32-bit word is read as one aligned load when the block starts
// on a 4-byte boundary and as two aligned loads joined by a funnel shift
// otherwise (every load stays inside the block's 210 bytes, or the block
// before it: a block 2 mod 4 never starts a matrix, whose base is
// 16-aligned). The weights are read once (no L1 allocation); the Q8_K
// activations through the read-only cache (every warp reads them).
#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace bh {

constexpr int Q6K_BYTES = 210;
constexpr int Q6K_WARPS = 8;
constexpr int Q6K_ROWS_PER_WARP = 4;  // 8 threads per row

__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// The 32-bit little-endian word at byte address p (p even): one aligned load,
// or two aligned loads and a funnel shift when p is 2 mod 4.
__device__ __forceinline__ uint32_t ld_word_a2(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    if ((a & 2) == 0) return ld_stream_u32(q);
    return __funnelshift_r(ld_stream_u32(q), ld_stream_u32(q + 1), 16);
}

// Sign-extended byte k (0..3) of a word.
__device__ __forceinline__ int sbyte(uint32_t w, int k) { return (int)(int8_t)(w >> (8 * k)); }

template <int NB>
__global__ void __launch_bounds__(Q6K_WARPS * 32) q6k_matvec_kernel(const uint8_t* __restrict__ W, int64_t N, int nb,
                                                                   const uint8_t* __restrict__ xq, int B,
                                                                   float* __restrict__ y) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int m = lane & 7;            // accumulator lane of this thread
    const int rg = lane >> 3;          // row of the warp's tile
    const int hsel = m >= 4 ? 1 : 0;   // which scale of a vector pair this lane uses
    const int64_t row = ((int64_t)blockIdx.x * Q6K_WARPS + warp) * Q6K_ROWS_PER_WARP + rg;
    const bool live = row < N;
    const uint8_t* wrow = W + (live ? row : 0) * (int64_t)nb * Q6K_BYTES;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    pdl_wait();
    for (int kb = 0; kb < nb; ++kb) {
        const uint8_t* blk = wrow + (int64_t)kb * Q6K_BYTES;
        // this lane's ql words (halves j = 0, 1; offsets 0 and 32), qh words
        uint32_t ql[2][2], qh[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            ql[j][0] = ld_word_a2(blk + 64 * j + 4 * m);
            ql[j][1] = ld_word_a2(blk + 64 * j + 32 + 4 * m);
            qh[j] = ld_word_a2(blk + 128 + 32 * j + 4 * m);
        }
        // scales: words 0..3 of the 16 int8 scales, and d
        uint32_t scw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) scw[k] = ld_word_a2(blk + 192 + 4 * k);
        // d (bytes 208..209): from the aligned word that holds it, so that no
        // load reaches past the block
        const bool odd = (reinterpret_cast<uintptr_t>(blk) & 2) != 0;
        const uint32_t dw = ld_stream_u32(reinterpret_cast<const uint32_t*>(blk + (odd ? 206 : 208)));
        const float xd = h2f((uint16_t)(odd ? (dw >> 16) : (dw & 0xffffu)));
        // the vector scale of this lane for vector is: scales[2 is + hsel]
        int vsc[8];
#pragma unroll
        for (int is = 0; is < 8; ++is) vsc[is] = sbyte(scw[(2 * is + hsel) >> 2], (2 * is + hsel) & 3);
        // the 6-bit codes of the 8 vectors (bytes 4m..4m+3 of each)
        uint32_t q[8];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const uint32_t lo = (x & 2) ? ((ql[j][x & 1] >> 4) & 0x0f0f0f0fu) : (ql[j][x & 1] & 0x0f0f0f0fu);
                q[4 * j + x] = lo | (((qh[j] >> (2 * x)) & 0x03030303u) << 4);
            }
        }
        // the offset term: bsums[2m], bsums[2m+1] against scales[2m], scales[2m+1]
        const int sc_a = sbyte(scw[(2 * m) >> 2], (2 * m) & 3), sc_b = sbyte(scw[(2 * m + 1) >> 2], (2 * m + 1) & 3);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint8_t* xb = xq + ((int64_t)b * nb + kb) * Q8K_BYTES;
            const int* a = reinterpret_cast<const int*>(xb + 4);
            int sumi = 0;
#pragma unroll
            for (int v = 0; v < 8; ++v) sumi += vsc[v] * dp4a((int)q[v], __ldg(a + 8 * v + m), 0);
            const uint32_t bs = (uint32_t)__ldg(reinterpret_cast<const int*>(xb + 260) + m);
            sumi -= ((int)(int16_t)(bs & 0xffffu) * sc_a + (int)(int16_t)(bs >> 16) * sc_b) << 5;
            const float d = __fmul_rn(__ldg(reinterpret_cast<const float*>(xb)), xd);
            acc[b] = __fmaf_rn(d, __int2float_rn(sumi), acc[b]);
        }
    }
    // hsum_float_8 (arch/x86/quants.c:43-49): ((a4+a0)+(a6+a2)) + ((a5+a1)+(a7+a3))
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const float t1 = __fadd_rn(acc[b], __shfl_xor_sync(0xffffffffu, acc[b], 4));
        const float t2 = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
        const float v = __fadd_rn(t2, __shfl_xor_sync(0xffffffffu, t2, 1));
        if (live && m == 0) y[(int64_t)b * N + row] = v;
    }
}

template <int NB>
static int launch_q6k_t(const uint8_t* W, int64_t N, int nb, const uint8_t* xq, int B, float* y, cudaStream_t s) {
    const int64_t rows_per_cta = (int64_t)Q6K_WARPS * Q6K_ROWS_PER_WARP;
    const int64_t grid = (N + rows_per_cta - 1) / rows_per_cta;
    q6k_matvec_kernel<NB><<<(unsigned)grid, Q6K_WARPS * 32, 0, s>>>(W, N, nb, xq, B, y);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

int launch_q6k_matvec(const uint8_t* W, int64_t N, int64_t K, const uint8_t* xq, int B, float* y, cudaStream_t s) {
    if (N < 1 || K < QK || K % QK || B < 1 || B > BH_MAX_BATCH || N > ((int64_t)1 << 31) / 4) return BH_EINVAL;
    const int nb = (int)(K / QK);
    switch (B) {
        case 1: return launch_q6k_t<1>(W, N, nb, xq, B, y, s);
        case 2: return launch_q6k_t<2>(W, N, nb, xq, B, y, s);
        case 3: return launch_q6k_t<3>(W, N, nb, xq, B, y, s);
        case 4: return launch_q6k_t<4>(W, N, nb, xq, B, y, s);
        case 5: return launch_q6k_t<5>(W, N, nb, xq, B, y, s);
        case 6: return launch_q6k_t<6>(W, N, nb, xq, B, y, s);
        case 7: return launch_q6k_t<7>(W, N, nb, xq, B, y, s);
        default: return launch_q6k_t<8>(W, N, nb, xq, B, y, s);
    }
}

}  // namespace bh

namespace {
inline bool aligned_to(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
}  // namespace

extern "C" int bh_q6k_matvec(bh_ctx* ctx, const void* W_q6k, int64_t N, int64_t K, const void* x_q8k, int B, float* y,
                             int fold, void* stream) {
    if (!ctx || !W_q6k || !x_q8k || !y || N < 1 || K < bh::QK || K % bh::QK || B < 1 || B > BH_MAX_BATCH)
        return BH_EINVAL;
    if (fold != BH_FOLD_X86) return BH_EINVAL;  // the x86 AVX2 fold only
    if (!aligned_to(W_q6k, 4) || !aligned_to(x_q8k, 4) || !aligned_to(y, 4)) return BH_EINVAL;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return BH_ENODEV;
    return bh::launch_q6k_matvec(static_cast<const uint8_t*>(W_q6k), N, K, static_cast<const uint8_t*>(x_q8k), B, y,
                                 static_cast<cudaStream_t>(stream));
}
