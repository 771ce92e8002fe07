// bh_ctx.cuh — the context object behind the opaque bh_ctx handle, and the
// internal launch planner shared by the C-ABI entry points.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <vector>
#include <cuda_runtime.h>

#include "bh_kernels.cuh"

// A mutex that copies as a fresh one (a context is copied only as a launch
// plan, which never touches the lock of the original).
struct bh_copyable_mutex {
    std::mutex m;
    bh_copyable_mutex() = default;
    bh_copyable_mutex(const bh_copyable_mutex&) {}
    bh_copyable_mutex& operator=(const bh_copyable_mutex&) { return *this; }
};

struct bh_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    int* d_status = nullptr;
    // scratch for host-buffer entry points and argmax candidates
    uint8_t* scratch = nullptr;
    size_t scratch_bytes = 0;
    // launch-shape tuning (bh_tune)
    int ctas_per_sm = 2;
    // bytes of one row's slice in a dense matvec stage, and in a routed-expert
    // one (BH_TUNE_STAGE_BYTES sets both); measured on B200, back-to-back
    // standalone launches: 1440 with one stage before the programmatic wait
    // beat 576 with the whole ring before it at every shape and batch of
    // configs 1 and 3 (4096x12288 batch 1: 11.0 against 13.6 us)
    int stage_bytes = 1440;
    int moe_stage_bytes = 576;
    int smem_cap_small = 100 * 1024;
    int small_act_bytes = 24 * 1024;
    int tpr_force = 0;  // threads per matvec row: 0 = planner's choice, else 4, 8 or 16
    // threads per row the planner takes at batch 1-2 for matrices with fewer
    // than two 8-row tiles per warp (4 for standalone launches; the decode
    // stack's plan sets 8)
    int tpr_narrow = 4;
    bool api_pdl = false;  // the C-ABI matvecs launch with programmatic dependent launch
    int sm_budget = 0;  // shared memory one matvec launch may hold per SM (0 = no limit)
    int prefill_stages = 1;  // ring stages per warp a matvec issues before its programmatic wait (0 = all, -1 = none)
    // decode stacks: bytes of the weights after a launch's own that it
    // prefetches into the L2 (-1: the stack's default)
    int64_t prefetch_bytes = -1;
    int64_t* trace = nullptr;  // timeline probe buffer (trace builds only)
    // argmax candidates of the LM-head entry point: [num_sms * 4][BH_MAX_BATCH]
    float* cand_val = nullptr;
    int32_t* cand_idx = nullptr;
    // routed-expert FFN scratch: grid-barrier words, gate|up and expert
    // outputs of every pair, routing
    uint8_t* moe_scratch = nullptr;
    size_t moe_scratch_bytes = 0;
    // Grid-barrier words of the cooperative MoE launches made through this
    // context (its own scratch and those of its MoE stacks). A CTA whose
    // bounded barrier wait ran out returns early and leaves its arrivals
    // counted, so bh_device_status zeroes every registered word when it finds
    // a timeout; until then later MoE results are not valid.
    bh_copyable_mutex barrier_mu;
    std::vector<void*> barrier_words;  // 256 bytes each
    // bound of the MoE grid-barrier wait in SM cycles (default ~1 s)
    long long barrier_wait_cycles = 1ll << 31;
};


namespace bh {
// Grid and shared-memory plan for one matvec launch (fills p's tiling
// fields); returns the grid size or a negative errno.
int plan_for(bh_ctx* ctx, MatvecParams& p, int grid_override, int fold);
// MatvecParams for a single-segment weight matrix.
MatvecParams base_params(bh_ctx* ctx, const void* W, int64_t N, int64_t K, int B, float* y);
// Grid-barrier words (256 bytes) that bh_device_status zeroes after a timeout.
void register_barrier_words(bh_ctx* ctx, void* words);
void unregister_barrier_words(bh_ctx* ctx, void* words);
// plan_for + launch.
int run_matvec(bh_ctx* ctx, MatvecParams& p, int fold, int src, int epi, cudaStream_t s, bool pdl);
// Plan and launch one routed-expert FFN batch (one cooperative launch; the
// PDL attribute only when pdl is set). p carries the shapes, routing source,
// h / gamma, the three banks, the scratch, out and the grid-barrier words.
int run_moe(bh_ctx* ctx, MoeParams& p, int fold, cudaStream_t s, bool pdl);
}  // namespace bh
