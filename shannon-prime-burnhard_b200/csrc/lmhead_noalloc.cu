// lmhead_noalloc.cu — the LM-head greedy pick for callers that cannot
// allocate device memory.
//
// Some embedders cannot call cudaMalloc at all: a caller running inside
// another runtime's memory pool, or one whose allocations are all made up
// front and then frozen (fixed-footprint serving processes), cannot let a
// library grab memory on a hot path, and cannot create a bh_ctx either
// (bh_init allocates). bh_q4k_lmhead_argmax_noalloc needs no context and
// allocates nothing: the per-CTA argmax candidates that bh_q4k_lmhead_argmax
// keeps in context memory live here in a file-scope device array instead.
//
//  - Size: NOALLOC_SCRATCH_BYTES (32 KiB) = 4096 candidate slots (value +
//    index); a launch needs grid x batch slots (at most 2368 on a 148-SM
//    B200 at batch 8). Larger requests are rejected with BH_EINVAL.
//  - Every GPU that loads the library holds the array until the process exits.
//  - Set-up: the first call on a device, with that device current, looks up
//    the array's device address with cudaGetSymbolAddress (host code must not
//    use the array's name as a pointer: it is a host-side stand-in). Make that
//    first call before any stream capture.
//  - Every call shares the array and it keeps the last call's contents.
//    Nothing in it needs to start at zero (each CTA writes its slots before
//    the finisher reads them), but calls that overlap on the GPU race on it:
//    serialize them (one stream, or events).
//  - Device-side failures: a second static word holds the status that the
//    kernels set when a bounded wait runs out. It is sticky: once set, every
//    later call writes -1 as its token, until bh_noalloc_status(1) reads and
//    clears it (the word starts at zero when the library loads).
#include <climits>
#include <mutex>

#include "bh_common.cuh"
#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace {

constexpr int NOALLOC_SLOTS = 4096;
constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)NOALLOC_SLOTS * (sizeof(float) + sizeof(int32_t));

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
static __device__ int g_noalloc_status;

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_scratch_dev[MAX_DEVICES];
int* g_status_dev[MAX_DEVICES];

// Device addresses of the scratch array and the status word on the current
// device (set-up on the first call per device).
int scratch_address(int device, unsigned char** out, int** status) {
    if (device < 0 || device >= MAX_DEVICES) return BH_ENODEV;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_dev[device]) {
        void* ptr = nullptr;
        void* sptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr ||
            cudaGetSymbolAddress(&sptr, g_noalloc_status) != cudaSuccess || !sptr) {
            cudaGetLastError();
            return BH_EIO;
        }
        g_status_dev[device] = static_cast<int*>(sptr);
        g_scratch_dev[device] = ptr;
    }
    *out = static_cast<unsigned char*>(g_scratch_dev[device]);
    *status = g_status_dev[device];
    return BH_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

extern "C" int bh_q4k_lmhead_argmax_noalloc(const void* W_q4k, int64_t N, int64_t K, const float* x, int B,
                                            float* logits_opt, int32_t* tok_out, float* max_opt, int fold,
                                            void* stream) {
    if (!W_q4k || !x || !tok_out || N < 1 || N > INT32_MAX || K < bh::QK || K % bh::QK != 0 || B < 1 ||
        B > BH_MAX_BATCH)
        return BH_EINVAL;
    if (fold != BH_FOLD_X86 && fold != BH_FOLD_GENERIC) return BH_EINVAL;
    if (!aligned(W_q4k, 16) || !aligned(x, 16) || !aligned(tok_out, 4) || (logits_opt && !aligned(logits_opt, 4)) ||
        (max_opt && !aligned(max_opt, 4)))
        return BH_EINVAL;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return BH_ENODEV;
    unsigned char* scratch = nullptr;
    int* status = nullptr;
    int rc = scratch_address(device, &scratch, &status);
    if (rc != BH_OK) return rc;

    // a context on the stack: launch tuning defaults, no device memory
    bh_ctx local;
    local.device = device;
    if (cudaDeviceGetAttribute(&local.num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
        return BH_ENODEV;
    bh::MatvecParams p = bh::base_params(&local, W_q4k, N, K, B, logits_opt);
    p.status = status;
    p.xf = x;
    const int grid = bh::plan_for(&local, p, 0, fold);
    if (grid < 0) return grid;
    if ((int64_t)grid * B > NOALLOC_SLOTS) return BH_EINVAL;  // more candidates than the static scratch holds
    p.cand_val = reinterpret_cast<float*>(scratch);
    p.cand_idx = reinterpret_cast<int32_t*>(scratch + (size_t)NOALLOC_SLOTS * sizeof(float));
    bh::LaunchOpts o;
    o.stream = static_cast<cudaStream_t>(stream);
    o.grid = grid;
    if ((rc = bh::launch_matvec(p, fold, bh::ACT_F32, bh::EPI_ARGMAX, o)) != BH_OK) return rc;
    return bh::launch_argmax_finish(p.cand_val, p.cand_idx, grid, B, tok_out, max_opt, o.stream, false, status);
}

extern "C" int bh_noalloc_status(int clear) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return BH_ENODEV;
    unsigned char* scratch = nullptr;
    int* status = nullptr;
    int rc = scratch_address(device, &scratch, &status);
    if (rc != BH_OK) return rc;
    // the word is read after every kernel queued on this device has finished
    if (cudaDeviceSynchronize() != cudaSuccess) return BH_EIO;
    int st = 0;
    if (cudaMemcpy(&st, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return BH_EIO;
    if (clear && st && cudaMemset(status, 0, sizeof(int)) != cudaSuccess) return BH_EIO;
    if (st == bh::ST_TIMEOUT) return BH_ETIMEDOUT;
    return st == bh::ST_OK ? BH_OK : BH_EINVAL;
}
