// bh_common.cuh — shared device helpers for the sm_100a Q4_K kernels.
//
// PTX wrappers (mbarrier, 1-D bulk async copy, programmatic dependent
// launch), the bounded-wait policy, and the exact-rounding helpers that the
// bit-exact paths rely on. Every kernel file is compiled with -fmad=false,
// so a*b+c is two roundings unless written as __fmaf_rn.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/bh_q4k.h"

namespace bh {

constexpr int QK = 256;           // values per super-block
constexpr int Q4K_BYTES = 144;    // block_q4_K (ggml-common.h:317-328)
constexpr int Q8K_BYTES = 292;    // block_q8_K (ggml-common.h:360-366)

// Device status word values (mirrors the negative errno codes of the C ABI).
constexpr int ST_OK = 0;
constexpr int ST_TIMEOUT = 1;     // a bounded wait ran out
constexpr int ST_BADARG = 2;      // a device-side argument check failed

// Bounded waits: ~2^31 SM cycles (about a second at B200 clocks).
constexpr long long WAIT_LIMIT_CYCLES = 1ll << 31;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity; false when the bound ran out.
// try_wait suspends the thread for a while on its own, so the clock is only
// consulted every 64 polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 0 && clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 2-D tensor copy global -> shared (cp.async.bulk.tensor, tile mode): the
// box at element coordinates (x, y) of the tensor map lands densely at dst;
// out-of-range elements are zero-filled. x * element size must be a multiple
// of 16 bytes.
__device__ __forceinline__ void tensor_g2s_2d(void* dst, const CUtensorMap* tmap, int x, int y, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 3-D tensor copy global -> shared (tile mode), coordinates (x, y, z); x * 8
// bytes must be a multiple of 16.
__device__ __forceinline__ void tensor_g2s_3d(void* dst, const CUtensorMap* tmap, int x, int y, int z, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bring [src, src + bytes) of this GPU's global memory into the L2 without
// waiting for it (cp.async.bulk.prefetch.L2, no multicast): a later load of
// those bytes hits the L2. src and bytes must be multiples of 16. The lines
// get the normal eviction priority, so they outlive the evict-first lines of
// the weight stream that is being consumed meanwhile.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Warp `wg` of `nw` warps issues its share of an L2 prefetch of `bytes`
// bytes at `base`: pieces of PREFETCH_PIECE bytes, piece i by warp i % nw
// (lane 0 issues; nothing waits on them).
constexpr uint32_t PREFETCH_PIECE = 32768;
__device__ __forceinline__ void prefetch_share(const uint8_t* base, int64_t bytes, int64_t wg, int64_t nw, int lane) {
    if (lane != 0 || !base || bytes <= 0) return;
    const int64_t pieces = (bytes + PREFETCH_PIECE - 1) / PREFETCH_PIECE;
    for (int64_t i = wg; i < pieces; i += nw) {
        const int64_t off = i * PREFETCH_PIECE;
        const int64_t n = bytes - off < (int64_t)PREFETCH_PIECE ? bytes - off : (int64_t)PREFETCH_PIECE;
        prefetch_l2(base + off, (uint32_t)(n & ~(int64_t)15));
    }
}

// Fetch a tensor map descriptor (generic address of the kernel parameter) ahead of the
// first copy that uses it.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Staged Q8_K activation block in shared memory (layout in q8k_device.cuh):
// lane m's codes at act_lane_off(m), then d and the paired bsums.
constexpr int ACT_D_OFF = 272;
constexpr int ACT_S_OFF = 288;
__host__ __device__ constexpr int act_lane_off(int m) { return 32 * m + (m >= 4 ? 16 : 0); }

// Small tensors every step reads again (norm weights, the KV cache) are
// loaded with an L2 evict-last hint, so the step's weight stream (loaded
// evict-first) does not push them out of the L2 between steps.
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ float4 ldg_f4_keep(const float* ptr, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(ptr), "l"(pol));
    return v;
}

// Programmatic dependent launch (no-ops when the launch did not opt in).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier among a subset of warps (id 1.. ; id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void set_status(int* status, int code) {
    if (status) atomicCAS(status, ST_OK, code);
}

// Round to nearest, ties to even, through the 1.5*2^23 bias — the integer
// rounding of ggml-quants.c:559-563, evaluated with a correctly rounded add.
// System-scope release store / reduction and acquire load (flags and
// counters that another GPU writes or reads over NVLink).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int round_biased(float v) {
    const float b = __fadd_rn(v, 12582912.f);
    return (__float_as_int(b) & 0x007fffff) - 0x00400000;
}

// Exact int -> float for |v| < 2^22 without the conversion unit: the
// integer is placed in the mantissa of 1.5 * 2^23 and the bias subtracted.
__device__ __forceinline__ float i2f_exact(int v) {
    return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.f);
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

}  // namespace bh
