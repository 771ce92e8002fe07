// peer_xchg.cu — the row-split LM head's greedy pick exchanged between the
// GPUs of one node through peer memory (NVLink), in the same kernel that
// reduces this GPU's per-CTA candidates: no NCCL call, no host round trip.
//
// Every rank owns a small mailbox in its own device memory: two banks (odd
// and even calls) of XCHG_MAX_WORLD slots of (value, global index) per batch
// column, then one flag word per slot. A rank's finish kernel reduces its candidates to (max, first index),
// stores that pair into slot `rank` of EVERY rank's mailbox (its own and the
// peers', mapped into this process through CUDA IPC), makes the stores
// visible system-wide, then sets the flag of slot `rank` in every mailbox to
// the call's epoch (release). It then waits, bounded, until all `world` flags
// of its own mailbox carry the epoch (acquire) and merges the slots in rank
// order (= row order): the maximum, first index among equals, as the
// reference's greedy loop over the whole vocabulary (engine.cpp:36-43).
//
// The epoch is a per-call counter supplied by the host (1, 2, 3, ...); a
// fresh mailbox is zeroed, so no flag matches before the first write. The
// wait gives up after WAIT_LIMIT_CYCLES (about a second) with ST_TIMEOUT in
// the status word; the host then reports BH_ETIMEDOUT.
#include <cstring>

#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace bh {

constexpr int XCHG_MAX_WORLD = 8;  // GPUs of one node

struct XchgSlot {
    float v[BH_MAX_BATCH];
    int32_t i[BH_MAX_BATCH];
};
// two banks, used by odd and even epochs: a rank can be at most one call ahead
// of another (it cannot finish a call before every rank has published in it),
// so a bank is never rewritten while a slower rank still reads it
constexpr size_t XCHG_BANK = sizeof(XchgSlot) * XCHG_MAX_WORLD + 4 * XCHG_MAX_WORLD;  // slots, then flags
constexpr size_t XCHG_FLAGS_OFF = sizeof(XchgSlot) * XCHG_MAX_WORLD;
constexpr size_t XCHG_BYTES = 2048;
static_assert(2 * XCHG_BANK <= XCHG_BYTES && XCHG_BANK % 16 == 0, "mailbox layout");

struct XchgParams {
    const float* cv;
    const int32_t* ci;
    int ncand, B;
    int64_t row_offset;
    int rank, world;
    uint8_t* box[XCHG_MAX_WORLD];  // every rank's mailbox as seen from this process (own at [rank])
    uint32_t epoch;
    const uint32_t* epoch_dev;  // non-null: the epoch is *epoch_dev + 1 (read after the programmatic wait)
    uint32_t* step_out;         // non-null: receives the epoch once the pick is merged
    int32_t* tok;
    float* val;
    int* status;
};

__global__ void __launch_bounds__(256) xchg_argmax_kernel(const XchgParams a) {
    pdl_wait();
    const uint32_t epoch = a.epoch_dev ? *reinterpret_cast<const volatile uint32_t*>(a.epoch_dev) + 1u : a.epoch;
    __shared__ float sv[8], bestv[BH_MAX_BATCH];
    __shared__ int si[8], besti[BH_MAX_BATCH];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // this GPU's pick per column, from the matvec's per-CTA candidates
    for (int b = 0; b < a.B; ++b) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = threadIdx.x; c < a.ncand; c += blockDim.x) {
            const float v = a.cv[c * a.B + b];
            const int i = a.ci[c * a.B + b];
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
            if (bi == 0x7fffffff) bi = 0;  // all candidates NaN: local row 0
            bestv[b] = bv;
            besti[b] = (int)(bi + a.row_offset);
        }
        __syncthreads();
    }
    if (threadIdx.x != 0) return;
    const size_t bank = (epoch & 1u) * XCHG_BANK;
    // publish: the pair into slot `rank` of every mailbox, then the flags
    for (int q = 0; q < a.world; ++q) {
        XchgSlot* s = reinterpret_cast<XchgSlot*>(a.box[q] + bank) + a.rank;
        for (int b = 0; b < a.B; ++b) {
            s->v[b] = bestv[b];
            s->i[b] = besti[b];
        }
    }
    __threadfence_system();
    for (int q = 0; q < a.world; ++q)
        st_release_sys(reinterpret_cast<uint32_t*>(a.box[q] + bank + XCHG_FLAGS_OFF) + a.rank, epoch);
    // collect every rank's slot from this GPU's own mailbox (bounded waits)
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.box[a.rank] + bank + XCHG_FLAGS_OFF);
    const long long t0 = clock64();
    bool ok = true;
    for (int r = 0; r < a.world && ok; ++r) {
        while (ld_acquire_sys(flags + r) != epoch) {
            // (gives up at once when an earlier wait of the context ran out)
            if (clock64() - t0 > WAIT_LIMIT_CYCLES || (a.epoch_dev && *reinterpret_cast<const volatile int*>(a.status))) {
                ok = false;
                set_status(a.status, ST_TIMEOUT);
                break;
            }
        }
    }
    const XchgSlot* own = reinterpret_cast<const XchgSlot*>(a.box[a.rank] + bank);
    for (int b = 0; b < a.B; ++b) {
        float bv = -INFINITY;
        int bi = 0;
        if (ok) {
            // ranks in row order: strict > keeps the earlier (lower) index
            bv = __ldcv(&own[0].v[b]);
            bi = __ldcv(&own[0].i[b]);
            for (int r = 1; r < a.world; ++r) {
                const float v = __ldcv(&own[r].v[b]);
                const int i = __ldcv(&own[r].i[b]);
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
        }
        a.tok[b] = ok ? bi : -1;
        if (a.val) a.val[b] = bv;
    }
    if (a.step_out) *a.step_out = epoch;
}

int launch_xchg_argmax(const float* cv, const int32_t* ci, int ncand, int B, int64_t row_offset, int rank, int world,
                       void* const* boxes, uint32_t epoch, int32_t* tok, float* val, int* status, cudaStream_t s,
                       const uint32_t* epoch_dev, uint32_t* step_out) {
    XchgParams a;
    a.cv = cv;
    a.ci = ci;
    a.ncand = ncand;
    a.B = B;
    a.row_offset = row_offset;
    a.rank = rank;
    a.world = world;
    for (int q = 0; q < XCHG_MAX_WORLD; ++q) a.box[q] = q < world ? static_cast<uint8_t*>(boxes[q]) : nullptr;
    a.epoch = epoch;
    a.epoch_dev = epoch_dev;
    a.step_out = step_out;
    a.tok = tok;
    a.val = val;
    a.status = status;
    xchg_argmax_kernel<<<1, 256, 0, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

// ---------------------------------------------------------------------------
// expert-parallel MoE: the owned pairs' expert outputs through peer memory,
// fused with the slot-order combine
// ---------------------------------------------------------------------------
// Each rank computed the expert outputs of the (token, slot) pairs whose
// expert it owns (bh_q4k_moe_ep, rows of its own dout). One CTA copies those
// rows into the receive buffer of every other rank (same row), publishes its
// flag in every rank's mailbox, waits (bounded) for every rank's flag in its
// own mailbox, then forms out exactly as bh_moe_combine: per token, the slots
// in order, fp32 product summed in double, each pair's row taken from its own
// dout when it owns the expert and from the receive buffer otherwise. Rows of
// a pair are written by exactly one rank, so the result is bit-identical to
// one GPU. Receive buffers and flags have two banks (odd / even epochs).
struct MoeXchgParams {
    const float* dout;              // this rank's expert outputs [T*k][n_embd]
    float* recv[XCHG_MAX_WORLD];    // every rank's receive bank of this epoch, own at [rank]
    uint8_t* box[XCHG_MAX_WORLD];   // every rank's flag mailbox
    const int32_t* sel;             // [T][k] selected experts
    const float* w;                 // [T][k] weights
    int T, k, n_embd, e_lo, e_hi, rank, world, residual;
    uint32_t epoch;
    float* out;
    int* status;
};

__global__ void __launch_bounds__(1024) moe_xchg_combine_kernel(const MoeXchgParams a) {
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    const int n4 = a.n_embd / 4, npair = a.T * a.k;
    for (int q = 0; q < npair; ++q) {
        const int e = __ldcg(a.sel + q);
        if (e < a.e_lo || e >= a.e_hi) continue;  // (the same q for every thread)
        const float4* src = reinterpret_cast<const float4*>(a.dout + (int64_t)q * a.n_embd);
        for (int r = 0; r < a.world; ++r) {
            if (r == a.rank) continue;
            float4* dst = reinterpret_cast<float4*>(a.recv[r] + (int64_t)q * a.n_embd);
            for (int i = tid; i < n4; i += blockDim.x) dst[i] = __ldcg(src + i);
        }
    }
    __syncthreads();
    if (tid == 0) {
        const size_t bank = (a.epoch & 1u) * XCHG_BANK;
        __threadfence_system();
        for (int r = 0; r < a.world; ++r)
            st_release_sys(reinterpret_cast<uint32_t*>(a.box[r] + bank + XCHG_FLAGS_OFF) + a.rank, a.epoch);
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.box[a.rank] + bank + XCHG_FLAGS_OFF);
        const long long t0 = clock64();
        int ok = 1;
        for (int r = 0; r < a.world && ok; ++r) {
            while (ld_acquire_sys(flags + r) != a.epoch) {
                if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
                    ok = 0;
                    set_status(a.status, ST_TIMEOUT);
                    break;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const float* recv = a.recv[a.rank];
    for (int idx = tid; idx < a.T * a.n_embd; idx += blockDim.x) {
        const int t = idx / a.n_embd, i = idx - t * a.n_embd;
        // ggml_mul (fp32 product) then ggml_sum_rows over the slots (double, in order)
        double acc = 0.0;
        for (int s = 0; s < a.k; ++s) {
            const int q = t * a.k + s;
            const int e = __ldcg(a.sel + q);
            const float* row = (e >= a.e_lo && e < a.e_hi) ? a.dout : recv;
            acc = __dadd_rn(acc, (double)__fmul_rn(__ldcv(row + (int64_t)q * a.n_embd + i), __ldcg(a.w + q)));
        }
        const float v = __double2float_rn(acc);
        a.out[idx] = a.residual ? __fadd_rn(a.out[idx], v) : v;
    }
}

}  // namespace bh

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {
inline bool aligned_to(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// the context's device current for the scope of a call
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};
}  // namespace

extern "C" {

size_t bh_xchg_mailbox_bytes(void) { return bh::XCHG_BYTES; }

int bh_xchg_mailbox_alloc(bh_ctx* ctx, void** mailbox) {
    if (!ctx || !mailbox) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    void* p = nullptr;
    if (cudaMalloc(&p, bh::XCHG_BYTES) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    if (cudaMemset(p, 0, bh::XCHG_BYTES) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return BH_EIO;
    }
    *mailbox = p;
    return BH_OK;
}

int bh_xchg_alloc(bh_ctx* ctx, size_t bytes, void** buf) {
    if (!ctx || !buf || bytes == 0) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return BH_EIO;
    }
    *buf = p;
    return BH_OK;
}

size_t bh_moe_xchg_recv_bytes(int n_embd) {
    return n_embd < 1 ? 0 : 2 * (size_t)bh::MOE_MAX_PAIRS * (size_t)n_embd * sizeof(float);
}

int bh_moe_ep_exchange_combine(bh_ctx* ctx, const float* dout_own, void* const* recv, void* const* mailboxes,
                               const int32_t* selected, const float* weights, int n_tok, int k, int n_embd,
                               int expert_lo, int expert_hi, int rank, int world, uint32_t epoch, float* out,
                               int residual, void* stream) {
    if (!ctx || !dout_own || !aligned_to(dout_own, 16) || !recv || !mailboxes || !selected || !weights || !out)
        return BH_EINVAL;
    if (n_tok < 1 || n_tok > bh::MOE_MAX_TOK || k < 1 || k > bh::MOE_MAX_K || n_embd < 4 || n_embd % 4 ||
        expert_lo < 0 || expert_hi < expert_lo || world < 1 || world > bh::XCHG_MAX_WORLD || rank < 0 ||
        rank >= world || epoch == 0)
        return BH_EINVAL;
    if (!aligned_to(selected, 4) || !aligned_to(weights, 4) || !aligned_to(out, 4)) return BH_EINVAL;
    for (int q = 0; q < world; ++q)
        if (!recv[q] || !aligned_to(recv[q], 256) || !mailboxes[q] || !aligned_to(mailboxes[q], 256))
            return BH_EINVAL;
    DeviceGuard g(ctx->device);
    bh::MoeXchgParams a;
    a.dout = dout_own;
    const size_t bank = (epoch & 1u) * (size_t)bh::MOE_MAX_PAIRS * (size_t)n_embd;  // floats
    for (int q = 0; q < bh::XCHG_MAX_WORLD; ++q) {
        a.recv[q] = q < world ? static_cast<float*>(recv[q]) + bank : nullptr;
        a.box[q] = q < world ? static_cast<uint8_t*>(mailboxes[q]) : nullptr;
    }
    a.sel = selected;
    a.w = weights;
    a.T = n_tok;
    a.k = k;
    a.n_embd = n_embd;
    a.e_lo = expert_lo;
    a.e_hi = expert_hi;
    a.rank = rank;
    a.world = world;
    a.residual = residual != 0;
    a.epoch = epoch;
    a.out = out;
    a.status = ctx->d_status;
    bh::moe_xchg_combine_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError() == cudaSuccess ? BH_OK : BH_EIO;
}

int bh_xchg_mailbox_free(bh_ctx* ctx, void* mailbox) {
    if (!ctx) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    return cudaFree(mailbox) == cudaSuccess ? BH_OK : BH_EIO;
}

int bh_xchg_ipc_handle(bh_ctx* ctx, void* mailbox, void* handle_out) {
    if (!ctx || !mailbox || !handle_out) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, mailbox) != cudaSuccess) return BH_EIO;
    std::memcpy(handle_out, &h, sizeof(h));
    return BH_OK;
}

int bh_xchg_ipc_open(bh_ctx* ctx, const void* handle, void** peer_mailbox) {
    if (!ctx || !handle || !peer_mailbox) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return BH_EIO;
    }
    *peer_mailbox = p;
    return BH_OK;
}

int bh_xchg_ipc_close(bh_ctx* ctx, void* peer_mailbox) {
    if (!ctx || !peer_mailbox) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    return cudaIpcCloseMemHandle(peer_mailbox) == cudaSuccess ? BH_OK : BH_EIO;
}

int bh_q4k_lmhead_argmax_tp(bh_ctx* ctx, const void* W_local, int64_t n_local, int64_t K, const float* x, int B,
                            int64_t row_offset, int rank, int world, void* const* mailboxes, uint32_t epoch,
                            int32_t* tok_out, float* max_opt, int fold, void* stream) {
    if (!ctx || !W_local || !aligned_to(W_local, 16) || !x || !aligned_to(x, 16) || !tok_out ||
        !aligned_to(tok_out, 4) || (max_opt && !aligned_to(max_opt, 4)))
        return BH_EINVAL;
    if (n_local < 1 || n_local > INT32_MAX || K < bh::QK || K % bh::QK || B < 1 || B > BH_MAX_BATCH) return BH_EINVAL;
    if (world < 1 || world > bh::XCHG_MAX_WORLD || rank < 0 || rank >= world || !mailboxes || epoch == 0 ||
        row_offset < 0 || row_offset + n_local > INT32_MAX)
        return BH_EINVAL;
    if (fold != BH_FOLD_X86 && fold != BH_FOLD_GENERIC) return BH_EINVAL;
    for (int q = 0; q < world; ++q)
        if (!mailboxes[q] || !aligned_to(mailboxes[q], 256)) return BH_EINVAL;
    DeviceGuard g(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bh::MatvecParams p = bh::base_params(ctx, W_local, n_local, K, B, nullptr);
    p.xf = x;
    p.cand_val = ctx->cand_val;
    p.cand_idx = ctx->cand_idx;
    const int grid = bh::plan_for(ctx, p, 0, fold);
    if (grid < 0) return grid;
    bh::LaunchOpts o;
    o.stream = s;
    o.grid = grid;
    int rc = bh::launch_matvec(p, fold, bh::ACT_F32, bh::EPI_ARGMAX, o);
    if (rc != BH_OK) return rc;
    return bh::launch_xchg_argmax(ctx->cand_val, ctx->cand_idx, grid, B, row_offset, rank, world, mailboxes, epoch,
                                  tok_out, max_opt, ctx->d_status, s);
}

}  // extern "C"
