// bh_kernels.cuh — host-side launch descriptors shared by the kernel files
// and the C-ABI layer.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "bh_common.cuh"

namespace bh {

// Function attributes (dynamic shared-memory limit, carveout) are per device:
// `done` keeps one bit per device on which `set` already ran for one kernel
// (a function-local static of that kernel's launcher). Safe from several host
// threads: two threads may both run `set` once, which is harmless. Returns
// true when the attributes hold on the current device.
template <class F>
inline bool attrs_on_device(std::atomic<uint64_t>& done, F&& set) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return true;
    if (!set()) return false;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return true;
}

// Where the matvec prologue takes its activations from.
enum ActSrc : int {
    ACT_Q8K = 0,          // GGML block_q8_K columns
    ACT_F32 = 1,          // fp32 columns, quantized to Q8_K in the prologue
    ACT_F32_RMSNORM = 2,  // fp32 h, x = h / sqrt(mean(h^2) + eps) * gamma, then Q8_K
};

// What the epilogue does with the dot product v of row r, column b.
enum Epilogue : int {
    EPI_STORE = 0,   // y[b*ldy + r] = v
    EPI_ADD = 1,     // y[b*ldy + r] += v   (residual add)
    EPI_ARGMAX = 2,  // y[b*ldy + r] = v, plus per-CTA (max, first index) candidates
    // Gate/up pairs: segment 0 holds the gate rows, segment 1 the up rows
    // (N = 2 * n_ff virtual rows; w[1] after w[0] in memory, 16-byte
    // distance). Virtual tile j of R rows is gate rows [j*R/2, (j+1)*R/2)
    // followed by the same up rows (one 3-D copy), so one warp has both
    // values of row i: y[b*ldy + i] = silu(gate_i) * up_i, i < n_ff.
    EPI_SWIGLU = 3,
};

// Row-split (tensor-parallel) decode over the GPUs of one node. The vectors
// that one launch produces in row slices and the next reads whole (attention
// output, h, SwiGLU output) are arrays of 64-bit (value, generation) pairs
// with a copy on every rank: the producing launch stores each of its rows as
// one pair into every rank's copy (its own and, over NVLink, the peers'),
// and the reading launch takes a pair once its generation is the one it
// expects (bounded polling, then ST_TIMEOUT). A 64-bit aligned store is
// single-copy atomic, so a matching generation carries its value: no fence,
// flag or counter, and the producer ends as soon as its stores are issued.
// generation = completed steps * gen_mul + the exchange's offset (>= 1); a
// buffer is rewritten only after every rank has read the previous
// generation (each rank's next producer of it depends on data every reader
// publishes after reading).
constexpr int TP_MAX_WORLD = 8;
struct TpLL {
    const uint64_t* x;                 // input pairs (null: the plain fp32 input)
    uint64_t* y_self;                  // this rank's output pairs (null: the plain fp32 output)
    uint64_t* y_peer[TP_MAX_WORLD];    // the peers' copies (same offsets), npeer of them
    int npeer;
    const uint32_t* step;              // completed steps of the stack
    uint32_t gen_mul, gen_in, gen_out;
};

__device__ __forceinline__ uint32_t tp_gen(const TpLL& ll, uint32_t off) {
    return *reinterpret_cast<const volatile uint32_t*>(ll.step) * ll.gen_mul + off;
}

__device__ __forceinline__ void st_pair(uint64_t* p, float v, uint32_t gen) {
    const uint64_t w = (uint64_t)__float_as_uint(v) | ((uint64_t)gen << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Store one output value as a pair into this rank's and every peer's copy.
__device__ __forceinline__ void tp_store(const TpLL& ll, int64_t i, float v, uint32_t gen) {
    st_pair(ll.y_self + i, v, gen);
    for (int q = 0; q < ll.npeer; ++q) st_pair(ll.y_peer[q] + i, v, gen);
}

__device__ __forceinline__ void ld_pairs2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Eight consecutive values (16-byte aligned pairs) once all carry generation
// gen; false when the bound ran out, or when the status word already holds
// an error (an earlier wait of the stack ran out: the exchange is broken and
// later waits give up at once instead of each spending the bound); the
// values are then whatever was read.
__device__ __forceinline__ bool tp_load8(const uint64_t* src, uint32_t gen, float (&v)[8], const int* status) {
    uint64_t w[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) ld_pairs2(src + 2 * k, w[2 * k], w[2 * k + 1]);
    bool ok = true;
    long long t0 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (ok && (uint32_t)(w[k] >> 32) != gen) {
            if (t0 == 0) t0 = clock64();
            for (uint32_t n = 1;; ++n) {
                uint64_t a, b;
                ld_pairs2(src + (k & ~1), a, b);
                w[k] = (k & 1) ? b : a;
                if ((uint32_t)(w[k] >> 32) == gen) break;
                if ((n & 63u) == 0 &&
                    (clock64() - t0 > WAIT_LIMIT_CYCLES || (status && *reinterpret_cast<const volatile int*>(status)))) {
                    ok = false;
                    break;
                }
            }
        }
        v[k] = __uint_as_float((uint32_t)w[k]);
    }
    return ok;
}

struct MatvecParams {
    // one 2-D tensor map per weight segment: 8-byte elements, rows of
    // nb*144 bytes, box = (row_stride/8) x MV_ROWS (filled in by the planner)
    CUtensorMap tmap[3];
    const uint8_t* w[3];   // up to three row segments of one virtual weight matrix
    int64_t seg_end[3];    // cumulative row ends of the segments; seg_end[2] == N
    int64_t N;
    int K, nb, B;
    const uint8_t* xq;     // ACT_Q8K: B x nb x 292 bytes
    const float* xf;       // fp32 sources (ACT_F32*)
    const float* gamma;    // ACT_F32_RMSNORM weights [K]
    float eps;
    float* y;
    int64_t ldy;
    int32_t* partials;     // optional exact integer partials [B][N][nb][9]
    float* cand_val;       // EPI_ARGMAX: [gridDim][B] per-CTA maxima
    int32_t* cand_idx;     // EPI_ARGMAX: [gridDim][B] first index of the maxima
    int* status;           // device status word
    int64_t* trace;        // timeline probe (builds with BH_TRACE only; else unused)
    // optional copy of the epilogue's values (null: none): EPI_ADD the sums
    // [B][ldy] it stores, EPI_SWIGLU the gate and up rows [B][2][ldy] before
    // the SwiGLU (the decode stack keeps its last layer's for parity checks)
    float* capture;
    // optional L2 prefetch of weights a later launch streams (null: none):
    // every warp issues its share once its own weight copies are all issued
    // (warps without rows right after the programmatic wait), so the HBM
    // stream continues through this launch's tail and the next one's start
    const uint8_t* pf_ptr;
    int64_t pf_bytes;
    // tiling, chosen on the host
    int rows_per_tile;     // rows of one warp stage: 32 / tpr
    int tpr;               // threads per row: 4 or 8
    int kc;                // super-blocks per pipeline stage
    int row_stride;        // shared-memory bytes per row of a stage
    int stage_bytes;       // rows_per_tile * row_stride (a multiple of 128)
    int stages;
    int prefill;           // stages per warp issued before the programmatic wait (0 = the whole ring, -1 = none)
    int act_off, ring_off, bar_off, smem_bytes;
    // row-split decode: input and output vectors as exchanged pairs
    TpLL ll;
};

struct LaunchOpts {
    cudaStream_t stream = nullptr;
    bool pdl = false;      // programmatic dependent launch attribute
    int grid = 0;          // 0 = one CTA per SM (capped by N)
};

#ifndef BH_MV_WARPS
#define BH_MV_WARPS 8
#endif
constexpr int MV_WARPS = BH_MV_WARPS;       // routed-expert kernel: warps per CTA
constexpr int MV_THREADS = MV_WARPS * 32;
// Dense matvec: warps per CTA for a batch of B columns. Batch 1-2 runs one
// CTA of 16 warps per SM (twice the warps to hide each warp's dependent
// per-block chain; ~100 registers a thread); larger batches hold more
// accumulators per thread and run 8-warp CTAs at 4 threads per row, or
// 16-warp CTAs at 8 threads per row for narrow matrices.
constexpr int DENSE_MAX_WARPS = 16;
#ifndef BH_DENSE_W12
#define BH_DENSE_W12 16
#endif
// At 8 or 16 threads per row a thread holds one reference lane, which leaves
// room for 16 warps at any batch (narrow matrices at batch 3-8 run so).
__host__ __device__ constexpr int dense_warps(int B, int tpr = 4) { return (B <= 2 || tpr >= 8) ? BH_DENSE_W12 : 8; }
// CTAs per SM a dense matvec kernel is compiled for: 8-warp CTAs at batch 1-2
// are kept within half the register file, so the next launch of a step can be
// resident beside them (and start its weight copies) while they finish.
__host__ __device__ constexpr int dense_min_blocks(int B, int tpr = 4) {
    return (B <= 2 && dense_warps(B, tpr) == 8) ? 2 : 1;
}
constexpr int MV_ROWS = 8;                  // largest tile (rows of one warp stage); segment boundaries align to it
constexpr int ACT_BLOCK_BYTES = 304;   // staged Q8_K block: 272 (q8, lane-padded) + 16 (d) + 16 (S)

// Routed-expert FFN (the stock MoE block of the reference, gate|up -> SwiGLU
// -> down -> weighted sum over the top-k slots), one token batch of B <= 8.
constexpr int MOE_MAX_TOK = 8;
constexpr int MOE_MAX_K = 8;
constexpr int MOE_MAX_PAIRS = MOE_MAX_TOK * MOE_MAX_K;
constexpr int MOE_MAX_EXPERT = 256;
constexpr int MOE_MAX_EMBD_BLOCKS = 64;  // n_embd <= 16384

struct MoeParams {
    CUtensorMap tmap[3];   // gate bank, up bank, down bank (2-D, 8-byte elements)
    const uint8_t* w[3];
    int n_expert, n_embd, n_ff, k, B;
    int norm_topk;         // renormalise the selected weights to sum 1
    const float* logits;   // [B][n_expert] router logits, or null: routing given in ids_in / w_in
    const int32_t* ids_in; // [B][k]
    const float* w_in;     // [B][k]
    int32_t* ids_out;      // [B][k] routing, written by CTA 0 (may be null)
    float* w_out;          // [B][k]
    const float* h;        // [B][n_embd] input
    const float* gamma;    // RMSNorm weight [n_embd], or null: h is used as is
    float eps;
    float* gu;             // [B*k][2*n_ff]: gate | up of pair (token t, slot s) at row t*k + s
    float* dout;           // [B*k][n_embd]: unweighted expert outputs of each pair
    float* out;            // [B][n_embd]: the weighted sum (stored, or added when residual)
    int residual;
    // layers run by one launch (each reads h after the previous one added
    // to it; needs residual): per-layer strides of the routing inputs and
    // outputs, the norm weight, and the banks (the tensor maps cover all
    // layers: expert e of layer l is bank row block l * n_expert + e)
    int n_layer;
    int64_t logits_ls, gamma_ls, route_ls;
    // expert parallelism: only experts [e_lo, e_hi) are computed, from banks
    // holding exactly those experts (bank row block = expert - e_lo); with
    // combine == 0 the launch stops after writing dout (the rows of pairs on
    // other experts are set to -0.0, so summing the dout of all ranks
    // reproduces every value exactly) and out is not touched
    int e_lo, e_hi, combine;
    unsigned int* gbar;    // grid barrier word (arrivals, generation << 16), zero before first use
    long long gbar_wait;   // bound of a grid-barrier wait, SM cycles
    int* status;
    int64_t* trace;        // timeline probe (builds with BH_TRACE only; else unused)
    // tiling, chosen on the host: both phases share one ring of `stages`
    // slots of slot_bytes per warp
    int kc_gu, stride_gu, stage_gu;   // gate|up phase (K = n_embd)
    int kc_dn, stride_dn, stage_dn;   // down phase (K = n_ff)
    int slot_bytes, stages, act_blocks;
    int act_off, ring_off, bar_off, smem_bytes;
};

// Plan the fused MoE layer launch for a shared-memory budget; returns 0 or a
// negative errno.
int moe_plan(MoeParams& p, int smem_cap, int stage_target);
// One routed-expert FFN batch in a single cooperative launch (grid CTAs, all
// co-resident; o.grid is clamped to what fits).
int launch_moe(const MoeParams& p, int fold, const LaunchOpts& o);
// Routing alone (one CTA): logits -> ids_out / w_out.
int launch_moe_route(const MoeParams& p, const LaunchOpts& o);
// out[t][i] (+)= (float) sum_s (double)(dout[t*k+s][i] * w[t][s]); with dout2
// the pair rows are dout + dout2 (disjoint owners, -0.0 elsewhere)
int launch_moe_combine(const float* dout, const float* w, int B, int k, int n_embd, float* out, bool residual,
                       const LaunchOpts& o, const float* dout2 = nullptr);
int encode_q4k_map(CUtensorMap* map, const void* base, int64_t rows, int nb, int row_stride, int box_rows);
int encode_q4k_pair_map(CUtensorMap* map, const void* gate, int64_t rows, int nb, int64_t dist, int row_stride,
                        int box_rows);
// Seeded normal fill (splitmix64 -> Box-Muller in double, the oracle's
// generator): out[i] = mean + std * z(seed, first + i).
int fill_normal(float* out, int64_t n, int64_t first, uint64_t seed, double mean, double stddev, cudaStream_t s);

// Fill tiling fields of p for the given grid; returns 0 or a negative errno.
int matvec_plan(MatvecParams& p, int grid, int smem_cap, int stage_target, int tpr);
int launch_matvec(const MatvecParams& p, int fold, int act_src, int epi, const LaunchOpts& o);

int launch_q8k_quantize(const float* x, int64_t K, int B, uint8_t* out, int* status, cudaStream_t s);
int launch_q4k_quantize(const float* w, int64_t N, int64_t K, uint8_t* out, cudaStream_t s);
int launch_q4k_dequantize(const uint8_t* w, int64_t N, int64_t K, float* out, cudaStream_t s);
// status (may be null): when the word is nonzero as the finisher runs (an
// earlier bounded wait ran out), every token is written as -1.
// The row-split LM head's pick merged across ranks through peer mailboxes
// (peer_xchg.cu); epoch_dev, when set, replaces epoch by *epoch_dev + 1 and
// step_out receives the epoch at the end (the decode stack's step counter).
int launch_xchg_argmax(const float* cv, const int32_t* ci, int ncand, int B, int64_t row_offset, int rank, int world,
                       void* const* boxes, uint32_t epoch, int32_t* tok, float* val, int* status, cudaStream_t s,
                       const uint32_t* epoch_dev = nullptr, uint32_t* step_out = nullptr);
int launch_argmax_finish(const float* cand_val, const int32_t* cand_idx, int ncand, int B,
                         int32_t* tok_out, float* val_out, cudaStream_t s, bool pdl, const int* status = nullptr);

}  // namespace bh
