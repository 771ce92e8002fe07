/*
 * bh_q4k.h — C ABI of the B200 (sm_100a) Q4_K x Q8_K decode hot path.
 *
 * Drop-in boundary for BurnHard's decode matvecs: dense projections, the LM
 * head and routed-expert FFNs. Plain C types only; no CUDA or torch types in
 * any signature (streams travel as void*, i.e. a cudaStream_t; NULL is the
 * CUDA default stream, as in the CUDA runtime).
 *
 * Conventions (follow the reference's C entry points):
 *  - Every call returns int: 0 on success, a negative errno on failure
 *    (burnhard_residue_matmul.c:93,122 and sp_crt.c:481-496 use the same
 *    0 / negative convention). Arguments are validated on the host before
 *    any launch; an invalid call launches nothing.
 *  - Pointers are DEVICE pointers unless the parameter name starts with
 *    host_. Device buffers are caller-allocated and caller-owned
 *    (burnhard_residue_matmul.h:18-19).
 *  - Layouts are GGML's: a Q4_K weight matrix of N rows and K columns is
 *    N rows of K/256 consecutive 144-byte block_q4_K (ggml-common.h:317-328);
 *    an activation column is K/256 consecutive 292-byte block_q8_K
 *    (ggml-common.h:360-366); outputs are GGML dst [N, B]: column b holds
 *    y[b*N .. b*N+N-1]. K must be a multiple of 256, 1 <= B <= 8,
 *    Q4_K weight pointers 16-byte aligned, Q8_K / fp32 pointers 4-byte aligned.
 *  - A context is bound to one device and is not re-entrant: one host thread
 *    at a time per context (the reference's CRT context is single-writer,
 *    sp_crt_dispatch.h:32-33). Kernels are asynchronous on the given stream.
 *  - fold selects the fp32 reduction order reproduced bit-for-bit:
 *    BH_FOLD_X86 = the reference's x86 AVX2 vec_dot (ggml-cpu/arch/x86/
 *    quants.c:1900-1983), BH_FOLD_GENERIC = its portable vec_dot
 *    (ggml-cpu/quants.c:645-718). Integer partials are identical for both.
 */
#ifndef BH_Q4K_H
#define BH_Q4K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BH_OK 0
#define BH_EIO (-5)
#define BH_ENOMEM (-12)
#define BH_ENODEV (-19)
#define BH_EINVAL (-22)
#define BH_ETIMEDOUT (-110)

#define BH_FOLD_X86 0
#define BH_FOLD_GENERIC 1

#define BH_QK 256
#define BH_Q4K_BLOCK_BYTES 144
#define BH_Q8K_BLOCK_BYTES 292
#define BH_MAX_BATCH 8

typedef struct bh_ctx bh_ctx;

/* Library version, (major << 16) | minor. */
int bh_version(void);
/* Static text for a status code. */
const char *bh_strerror(int code);

/* Create / destroy a context on CUDA device `device` (sp_crt_dispatch.h:30-33,
 * 73-76: one context per engine, created at init, freed at shutdown). */
int bh_init(int device, bh_ctx **out);
int bh_free(bh_ctx *ctx);
/* The CUDA device ordinal of a context (or BH_EINVAL). */
int bh_ctx_device(bh_ctx *ctx);
/* Synchronize the context's device and report (and optionally clear) the
 * device-side status word that kernels set when a bounded wait runs out:
 * 0, or BH_ETIMEDOUT / BH_EINVAL. A routed-expert launch whose grid-barrier
 * wait ran out leaves that barrier's arrival count behind; clearing a timeout
 * also resets every grid barrier of the context and of its MoE stacks, and
 * MoE results computed between the timeout and that clear are not valid. */
int bh_device_status(bh_ctx *ctx, int clear);

/* Launch-shape tuning of a context (no effect on results): keys below.
 * BH_TUNE_CTAS_PER_SM: matvec CTAs per SM when the staged activations are
 *   small (batch x K/256 x 304 bytes <= 24 KiB), 1..4 (default 2);
 * BH_TUNE_STAGE_BYTES: bytes of one row's slice in a weight pipeline stage
 *   (rounded down to whole 144-byte blocks, shrunk until 2 stages fit),
 *   144..65536 (default 1440 for the dense matvecs, 576 for the routed
 *   experts; the key sets both); BH_TUNE_SMEM_CAP: shared-memory budget of a matvec CTA
 *   whose staged activations are small, 32768..204800 (default 102400). */
#define BH_TUNE_CTAS_PER_SM 1
#define BH_TUNE_STAGE_BYTES 2
#define BH_TUNE_SMEM_CAP 3
/* BH_TUNE_TPR: threads working one matvec row, 0 = the planner's choice
 * (4, and 8 for narrow matrices at batch 3-8; in the decode stack's plan 8
 * for the layer matrices), or 4 / 8 / 16 to force it (16: batch <= 2 with
 * BH_FOLD_X86 and no partials, else 8); results are identical either way. */
#define BH_TUNE_TPR 4
/* BH_TUNE_SM_BUDGET: shared memory (bytes) one matvec launch may occupy per
 * SM, 0 = no limit (default) or 48 KiB..228 KiB; below the SM's capacity the
 * next launch of a step can become resident early and start streaming its
 * weights while this one finishes. */
#define BH_TUNE_SM_BUDGET 5
/* BH_TUNE_SMALL_ACT: largest staged activation size (bytes, 0..128 KiB,
 * default 24 KiB) for which a matvec may run several CTAs per SM. */
#define BH_TUNE_SMALL_ACT 7
/* BH_TUNE_PREFILL: ring stages per warp a matvec issues before its
 * programmatic-launch wait, -1..8 (default 1; 0: the whole ring; -1: none);
 * the rest go out right after the activation loads that follow the wait. */
#define BH_TUNE_PREFILL 8
/* BH_TUNE_BARRIER_WAIT: log2 of the SM cycles a routed-expert grid barrier
 * waits before it gives up and reports BH_ETIMEDOUT, 16..31 (default 31,
 * about a second). */
#define BH_TUNE_BARRIER_WAIT 9
/* BH_TUNE_PREFETCH_MB: decode stacks created after the call prefetch into
 * the L2, from each launch, this many MiB of the weights the step streams
 * next (0 = off, -1 = the stack's default, at most 120). */
#define BH_TUNE_PREFETCH_MB 10
/* BH_TUNE_PDL: 1 launches the context's matvecs (bh_q4k_matvec,
 * bh_q4k_matvec_f32, bh_q4k_mul_mat_host, bh_q4k_lmhead_argmax) with the
 * programmatic-dependent-launch attribute: a matvec that follows another
 * kernel on the stream starts streaming its weights (and RMSNorm weights)
 * before that kernel ends, and reads its activations and writes its output
 * only after it. Only for sequences in which the kernel just before does not
 * write those weights. 0 (default): plain launches. */
#define BH_TUNE_PDL 11
int bh_tune(bh_ctx *ctx, int key, int value);

/* fp32 activations [B][K] -> B columns of Q8_K, byte-identical to
 * quantize_row_q8_K_ref (ggml-quants.c:2692-2729); replaces the CPU
 * backend's from_float step (ggml-cpu.c:1322-1333). All-zero blocks get
 * d = 0, qs = 0 and bsums = 0. */
int bh_q8k_quantize(bh_ctx *ctx, const float *x, int64_t K, int B, void *x_q8k, void *stream);

/* y[b*N + r] = W_q4k[r] . x_q8k[b] — the Q4_K x Q8_K matvec, batch 1..8.
 * Replaces the row loop of ggml_compute_forward_mul_mat (ggml-cpu.c:1151-1234)
 * over ggml_vec_dot_q4_K_q8_K. partials_opt (may be NULL) receives the exact
 * integer partials, int32 [B][N][K/256][9]: entries 0..7 are the unscaled
 * sub-block sums sum(q4*q8) over 32 values, entry 8 is the min term
 * sum_j min6_j * (bsums[2j] + bsums[2j+1]). */
int bh_q4k_matvec(bh_ctx *ctx, const void *W_q4k, int64_t N, int64_t K, const void *x_q8k, int B,
                  float *y, int32_t *partials_opt, int fold, void *stream);

/* Same product from fp32 activations [B][K]: the Q8_K quantization runs in
 * the matvec kernel's prologue (bit-identical to bh_q8k_quantize followed by
 * bh_q4k_matvec). This is ggml_mul_mat's contract for a Q4_K src0 and an
 * f32 src1 (ggml-cpu.c:1241-1439). */
int bh_q4k_matvec_f32(bh_ctx *ctx, const void *W_q4k, int64_t N, int64_t K, const float *x, int B,
                      float *y, int fold, void *stream);

/* y[b*N + r] = W_q6k[r] . x_q8k[b] for Q6_K weights (210-byte block_q6_K,
 * ggml-common.h:352-357: the matrices a Q4_K_M model file keeps in 6 bits),
 * batch 1..8, bit-identical to the x86 AVX2 ggml_vec_dot_q6_K_q8_K
 * (ggml-cpu/arch/x86/quants.c:2288-2370); fold must be BH_FOLD_X86. W_q6k is
 * 16-byte aligned (its blocks are then 2-byte aligned, as in a GGUF file). */
int bh_q6k_matvec(bh_ctx *ctx, const void *W_q6k, int64_t N, int64_t K, const void *x_q8k, int B, float *y,
                  int fold, void *stream);

/* fp32 weights [N][K] -> Q4_K, byte-identical to quantize_row_q4_K_ref
 * (ggml-quants.c:1395-1465) evaluated without FMA contraction; the
 * offline weight-prep step of ggml_quantize_chunk (ggml-quants.c:1564-1576). */
int bh_q4k_quantize(bh_ctx *ctx, const float *w, int64_t N, int64_t K, void *W_q4k, void *stream);

/* Q4_K -> fp32 [N][K], bit-identical to dequantize_row_q4_K
 * (ggml-quants.c:1467-1489). */
int bh_q4k_dequantize(bh_ctx *ctx, const void *W_q4k, int64_t N, int64_t K, float *w, void *stream);

/* Host-buffer form of the matvec, the call a CPU caller of ggml_mul_mat makes:
 * host_x fp32 [B][K] is copied in, quantized, multiplied by the device-resident
 * W_q4k, and host_y [B][N] is copied back before returning. Uses scratch
 * buffers owned by the context. */
int bh_q4k_mul_mat_host(bh_ctx *ctx, const void *W_q4k, int64_t N, int64_t K, const float *host_x,
                        int B, float *host_y, int fold);

/* LM head with the engine's greedy pick: logits = W_q4k . x for fp32
 * activations x [B][K] (quantized to Q8_K in the prologue), then
 * tok_out[b] = the first index of the maximum of column b, exactly
 * argmax() of desktop/engine/src/engine.cpp:36-43 (strict >, first wins).
 * logits_opt [B][N] and max_opt [B] may be NULL. The per-CTA argmax
 * candidates live in a buffer the context allocated at bh_init. */
int bh_q4k_lmhead_argmax(bh_ctx *ctx, const void *W_q4k, int64_t N, int64_t K, const float *x, int B,
                         float *logits_opt, int32_t *tok_out, float *max_opt, int fold, void *stream);

/* The same greedy LM-head pick for callers that cannot allocate device
 * memory (and so cannot create a bh_ctx): no context, no allocation. The
 * per-CTA argmax candidates live in a 32 KiB static device array of the
 * library (4096 slots; a launch needs grid x B of them, at most 2368 on a
 * 148-SM B200, larger requests return BH_EINVAL). The first call on a device
 * looks up that array's address (cudaGetSymbolAddress) and must come before
 * any stream capture. Calls share the array: calls that overlap on the GPU
 * race, so serialize them. Runs on the current device. No counterpart in the
 * reference.
 * Device-side failures (a bounded weight-copy wait that ran out) cannot be
 * returned by the call itself, which returns before the kernels run: they set
 * a second static status word, after which the call's tokens (and those of
 * every later call until the word is cleared) are written as -1.
 * bh_noalloc_status synchronizes the current device and returns that word as
 * BH_OK / BH_ETIMEDOUT, clearing it when clear != 0. */
int bh_q4k_lmhead_argmax_noalloc(const void *W_q4k, int64_t N, int64_t K, const float *x, int B,
                                 float *logits_opt, int32_t *tok_out, float *max_opt, int fold, void *stream);
int bh_noalloc_status(int clear);

/* Row-split (tensor-parallel) LM head over the GPUs of one node, one process
 * per GPU, with the greedy pick exchanged through peer memory instead of a
 * collective library call (the reference's LM head and argmax,
 * forward.cpp:3413 and engine.cpp:36-43, split by rows). Each rank owns a
 * mailbox (bh_xchg_mailbox_alloc, zeroed, XCHG bytes) and maps the peers'
 * mailboxes into its process with CUDA IPC (bh_xchg_ipc_handle on the owner,
 * the 64-byte handle passed by the caller, bh_xchg_ipc_open on the others).
 * bh_q4k_lmhead_argmax_tp computes this rank's rows [row_offset, row_offset +
 * n_local) and, in the kernel that reduces them, stores its (max, first index)
 * into every rank's mailbox, then waits (bounded, about a second) for all
 * ranks' pairs in its own mailbox and merges them in rank order: tok_out is
 * the global token on every rank, identical to one GPU over all rows.
 * mailboxes[q] is rank q's mailbox as seen from this process (own at [rank]);
 * epoch is the call's number, 1, 2, 3, ..., the same on every rank. A rank
 * that does not arrive makes the others return BH_ETIMEDOUT (tok_out = -1)
 * after the wait; calls of one group must not overlap. */
size_t bh_xchg_mailbox_bytes(void);
int bh_xchg_mailbox_alloc(bh_ctx *ctx, void **mailbox);
int bh_xchg_mailbox_free(bh_ctx *ctx, void *mailbox); /* also frees bh_xchg_alloc buffers */
int bh_xchg_ipc_handle(bh_ctx *ctx, void *mailbox, void *handle_out /* 64 bytes */);
int bh_xchg_ipc_open(bh_ctx *ctx, const void *handle, void **peer_mailbox);
int bh_xchg_ipc_close(bh_ctx *ctx, void *peer_mailbox);
int bh_q4k_lmhead_argmax_tp(bh_ctx *ctx, const void *W_local, int64_t n_local, int64_t K, const float *x, int B,
                            int64_t row_offset, int rank, int world, void *const *mailboxes, uint32_t epoch,
                            int32_t *tok_out, float *max_opt, int fold, void *stream);

/* The expert-parallel MoE exchange over peer memory instead of an
 * all-reduce (the other half of bh_q4k_moe_ep + bh_moe_combine): after
 * bh_q4k_moe_ep wrote this rank's pairs into dout_own, one kernel copies
 * those rows into every other rank's receive buffer, publishes this rank's
 * flag (epoch) in every rank's mailbox, waits (bounded, about a second, then
 * BH_ETIMEDOUT) for all ranks' flags in its own, and forms out as
 * bh_moe_combine does, each pair's row from dout_own when this rank owns
 * the expert and from the receive buffer otherwise: bit-identical to one GPU.
 * recv[q] / mailboxes[q]: rank q's receive buffer (bh_xchg_alloc of
 * bh_moe_xchg_recv_bytes(n_embd) bytes, two banks for odd and even epochs) and
 * mailbox as seen from this process (own at [rank]), mapped with
 * bh_xchg_ipc_open; epoch as for bh_q4k_lmhead_argmax_tp. */
int bh_xchg_alloc(bh_ctx *ctx, size_t bytes, void **buf);
size_t bh_moe_xchg_recv_bytes(int n_embd);
int bh_moe_ep_exchange_combine(bh_ctx *ctx, const float *dout_own, void *const *recv, void *const *mailboxes,
                               const int32_t *selected, const float *weights, int n_tok, int k, int n_embd,
                               int expert_lo, int expert_hi, int rank, int world, uint32_t epoch, float *out,
                               int residual, void *stream);

/* ------------------------------------------------------------------------
 * Decode block stack: the caller of the matvec in the reference engine's
 * per-token step (desktop/engine/src/forward.cpp:2663-2854 build_block_decode,
 * LM head :3413, argmax engine.cpp:36-43), for one sequence at batch 1, with
 * random-init (seeded N(0, 0.02)) Q4_K weights generated on the device.
 * Per layer: RMSNorm -> fused Q|K|V matvec -> q/k RMSNorm, NeoX RoPE, KV
 * append, GQA softmax attention -> O matvec + residual -> RMSNorm -> fused
 * gate|up matvec -> SiLU(gate)*up -> down matvec + residual; then RMSNorm ->
 * LM head -> argmax. The whole step is one CUDA graph.
 * ------------------------------------------------------------------------ */
typedef struct bh_stack bh_stack;
typedef struct bh_stack_config {
    int n_layer;      /* 36 for the Qwen3-8B shape */
    int n_embd;       /* 4096 */
    int n_head;       /* 32 query heads */
    int n_head_kv;    /* 8 KV heads */
    int head_dim;     /* 128 */
    int n_ff;         /* 12288 */
    int n_vocab;      /* 151936 */
    int n_ctx;        /* KV cache positions */
    float rms_eps;    /* 1e-6 */
    float rope_theta; /* 1e6 */
} bh_stack_config;

/* tensor ids for bh_stack_tensor */
#define BH_W_Q 0
#define BH_W_K 1
#define BH_W_V 2
#define BH_W_O 3
#define BH_W_GATE 4
#define BH_W_UP 5
#define BH_W_DOWN 6
#define BH_W_PER_LAYER 7
#define BH_W_OUTPUT 7
#define BH_T_ATTN_NORM 8
#define BH_T_FFN_NORM 9
#define BH_T_Q_NORM 10
#define BH_T_K_NORM 11
#define BH_T_OUT_NORM 12
#define BH_T_K_CACHE 13
#define BH_T_V_CACHE 14
#define BH_T_LOGITS 15
#define BH_T_HIDDEN 16
/* the last layer's activations of the last step: q|k|v as projected (before
 * the per-head norm and RoPE), and the attention output [n_head * head_dim] */
#define BH_T_QKV 17
#define BH_T_ATTN 18
/* the last layer's hidden state after the O projection and its residual add,
 * its gate | up rows before the SwiGLU [2 * n_ff], and silu(gate) * up [n_ff]
 * (the down projection's input) */
#define BH_T_H_ATTN 19
#define BH_T_GATE_UP 20
#define BH_T_FFN_ACT 21

/* The Qwen3-8B-shaped defaults (36 x 4096, 32/8 heads of 128, FFN 12288,
 * vocab 151936, 128 KV positions). */
void bh_stack_default_config(bh_stack_config *cfg);
/* Allocate the stack on ctx's device and generate its weights from seed. */
int bh_stack_create(bh_ctx *ctx, const bh_stack_config *cfg, uint64_t seed, bh_stack **out);
int bh_stack_free(bh_stack *st);
/* Position (0 <= pos < n_ctx) at which the next token is decoded; attention
 * covers positions 0..pos. */
int bh_stack_set_pos(bh_stack *st, int pos);
/* Seeded N(0, 1) K/V history for positions [0, n_pos) of every layer. */
int bh_stack_fill_kv(bh_stack *st, int n_pos, uint64_t seed);
/* One decode step from the device embedding x [n_embd]; the next token id
 * is written to device tok_out. Asynchronous on stream. */
int bh_stack_decode(bh_stack *st, const float *x, int32_t *tok_out, void *stream);
/* The same step from host memory: host_x is copied in, the step runs, and
 * the token is copied back before returning. */
int bh_stack_decode_host(bh_stack *st, const float *host_x, int32_t *host_tok);
/* Bytes of all Q4_K weights, algorithmic bytes of one step (weights plus
 * activations read and outputs written by the matvecs) and kernel launches
 * per step (on a row split: this rank's). */
int bh_stack_info(bh_stack *st, int64_t *weight_bytes, int64_t *step_bytes, int64_t *launches);
/* Average device time of one op of the step (CUDA events around reps
 * eager repetitions over all layers on the stack's stream, launched as
 * inside the step: the same launch parameters, programmatic dependent
 * launch), and its algorithmic bytes per launch.
 * The state it leaves (hidden, caches) is scratch: reset x / pos after it. */
#define BH_OP_QKV 0
#define BH_OP_O 1
#define BH_OP_GATE_UP 2
#define BH_OP_DOWN 3
#define BH_OP_LMHEAD 4
#define BH_OP_ATTN 5
int bh_stack_time_op(bh_stack *st, int op, int reps, float *avg_ms, int64_t *bytes_per_launch);
/* Device pointer and shape of one tensor (ids above); Q4_K matrices are
 * rows x cols in values, the rest fp32. */
int bh_stack_tensor(bh_stack *st, int layer, int which, void **ptr, int64_t *rows, int64_t *cols);

/* Row-split (tensor-parallel) decode over `world` GPUs of one node, one
 * process (and one context) per GPU. Rank r holds query heads
 * [r n_head / world, ...) with their KV heads, rows [r n_embd / world, ...)
 * of O and down, [r n_ff / world, ...) of gate and up, and an even share of
 * the LM head's rows, generated from the same seed as the one-GPU stack (the
 * same bytes for the same rows). Every matvec output row is computed whole
 * on one rank, so tokens and hidden states equal one GPU's bit for bit.
 * world in 1..8 dividing n_head_kv, n_embd / 8 and n_ff / 8; world 1 is
 * bh_stack_create. The launches that produce a vector the next launch reads
 * whole (attention output, h after O and after down, the SwiGLU output)
 * store each row as a 64-bit (value, generation) pair into every rank's copy
 * (over NVLink for the peers); the reading launch polls for the
 * generation it expects (bounded, about a second: then BH_ETIMEDOUT through
 * bh_device_status and the stack must be recreated). The LM head's pick is merged through peer mailboxes. Replaces
 * the reference's single-device path through forward.cpp:2706-2854 and the
 * NCCL all-gather of ggml-cuda.cu:1216. */
int bh_stack_create_tp(bh_ctx *ctx, const bh_stack_config *cfg, uint64_t seed, int rank, int world,
                       bh_stack **out);
/* CUDA IPC handle (64 bytes) of this rank's exchange region. */
int bh_stack_tp_handle(bh_stack *st, void *handle_out);
/* Map the peers' exchange regions: handles = world x 64 bytes in rank order
 * (this rank's own entry is ignored). Decoding needs it when world > 1. */
int bh_stack_tp_connect(bh_stack *st, const void *handles);
/* Rank, world and the owned ranges as (first, count) pairs: query heads, KV
 * heads, O / down rows, gate / up rows, LM head rows (10 int64). */
int bh_stack_tp_info(bh_stack *st, int *rank, int *world, int64_t *row_ranges);
/* On a row split: bh_stack_free after every rank's last decode has
 * completed (a host barrier), since the peers store into this rank's
 * exchange region; bh_stack_time_op is for one GPU only (BH_EINVAL); the
 * exchanged vectors (BH_T_HIDDEN, BH_T_ATTN, BH_T_FFN_ACT) are 64-bit
 * (fp32 value, generation) pairs, value in the low word (cols = 2 x n). */

/* ------------------------------------------------------------------------
 * The native engine's dense-matmul hook (forward_native.h:115-119,
 * mm_dispatch_fn_t; called by weight_matmul, forward_native.cpp:102-118).
 * The hook receives the fp16 copy of a weight, used here only as a key: the
 * engine registers at bind time the device Q4_K bytes (N rows x K, the GGUF
 * layout) of the same weight under that key. bh_mm_dispatch then computes
 * out[m][n] = W_q4k[n] . lhs[m] for host lhs [M][K] / out [M][N] with lhs
 * quantized to Q8_K and the x86 fold (ggml's own Q4_K matmul, bit for bit),
 * M in chunks of 8. It returns non-zero for a key that was not registered
 * or a shape that differs from the registration, and the engine falls
 * through to its CPU matmul as without a hook. Pass bh_mm_dispatch as
 * mm_dispatch and the registry as mm_dispatch_userdata.
 * ------------------------------------------------------------------------ */
typedef struct bh_mm_registry bh_mm_registry;
int bh_mm_registry_create(bh_ctx *ctx, bh_mm_registry **out);
int bh_mm_registry_add(bh_mm_registry *reg, const void *W_fp16_key, const void *W_q4k, int N, int K);
int bh_mm_registry_free(bh_mm_registry *reg);
int bh_mm_dispatch(void *userdata, const float *lhs, const uint16_t *W_fp16, int M, int K, int N, float *out);

/* ------------------------------------------------------------------------
 * NCCL communicators from C (tp_comm.cu). A communicator is a void*
 * (ncclComm_t). Creation is non-blocking (ncclCommInitRankConfig with
 * blocking = 0) and every wait is polled against timeout_ms of wall clock
 * (ncclCommGetAsyncError, cudaStreamQuery); when it runs out the
 * communicator is aborted (ncclCommAbort) and the call returns BH_ETIMEDOUT:
 * a rank that never joins or stops does not hang the others. NCCL is opened
 * at run time ($BH_NCCL_LIB, else libnccl.so.2); without it the calls return
 * BH_ENODEV.
 * ------------------------------------------------------------------------ */
/* ncclGetUniqueId on one rank; the 128 bytes reach the others through the
 * caller's own channel. */
int bh_tp_unique_id(void *id_out);
/* Join rank `rank` of `world` on `device` (-1: the current device). */
int bh_tp_comm_init(int device, const void *unique_id, int world, int rank, int timeout_ms, void **comm_out);
int bh_tp_comm_abort(void *comm);
/* ncclCommFinalize, bounded, then ncclCommDestroy (aborted on timeout). */
int bh_tp_comm_free(void *comm, int timeout_ms);
int bh_tp_comm_info(void *comm, int *rank, int *world);
/* recv [world][bytes_per_rank] <- every rank's send, completed on stream
 * before returning. */
int bh_tp_allgather(void *comm, const void *send, void *recv, size_t bytes_per_rank, void *stream, int timeout_ms);
/* buf <- the elementwise sum over ranks (the expert-parallel MoE's exchange:
 * bh_q4k_moe_ep writes -0.0 in the rows it does not own, so each sum has one
 * nonzero term and equals one GPU's value), completed before returning. */
int bh_tp_allreduce_sum_f32(void *comm, float *buf, size_t count, void *stream, int timeout_ms);
/* bh_stack_tp_connect with the handles all-gathered over comm (whose rank
 * and size must be the stack's). */
int bh_stack_tp_connect_comm(bh_stack *st, void *comm, int timeout_ms);

/* ------------------------------------------------------------------------
 * Routed-expert FFN (MoE): the stock block of desktop/engine/src/forward.cpp
 * :1001-1118 (ggml_soft_max -> ggml_top_k -> ggml_get_rows -> renormalise,
 * then three ggml_mul_mat_id + ggml_silu + ggml_mul + weighted sum) and the
 * BURN_MOE custom op that replaces its expert half (burn_moe_op.h:47-59,
 * burn_moe_op.cpp:202-372). At most 8 tokens per call, k <= 8 selected
 * experts per token, n_expert <= 256; n_embd and n_ff multiples of 256,
 * n_embd <= 16384.
 * ------------------------------------------------------------------------ */

/* Router of n_tok tokens from logits [n_tok][n_expert]: probabilities by
 * soft_max (max subtracted, exp, sum in double of per-8 fp32 partial sums,
 * scaled by (float)(1/sum)); the k largest in descending order with slots 0
 * and 1 swapped, as ggml_top_k writes them (ggml-cpu/ops.cpp:8157-8194;
 * equal probabilities lower index first); their probabilities, divided by
 * their double sum when norm_topk != 0. selected_out / weights_out are
 * device [n_tok][k]. exp is the reference's AVX2 ggml_v_expf, lane for lane
 * (ggml-cpu/vec.h), so probabilities and weights equal the reference's. */
int bh_moe_route(bh_ctx *ctx, const float *logits, int n_tok, int n_expert, int k, int norm_topk,
                 int32_t *selected_out, float *weights_out, void *stream);

/* out[t] = sum over slots s, in order, of w[t][s] * down_e(silu(gate_e . x_t) * (up_e . x_t)),
 * e = selected[t][s], for cur [n_tok][n_embd] fp32 (each column quantized
 * to Q8_K; silu(gate) * up quantized again for down), accumulated in double
 * and rounded once (ggml_mul then ggml_sum_rows). Banks are GGML's bundled
 * expert tensors in block_q4_K rows: gate_exps / up_exps [n_expert][n_ff][n_embd],
 * down_exps [n_expert][n_embd][n_ff]. Routing is either given (selected,
 * weights: device [n_tok][k], BURN_MOE's inputs) or computed from
 * router_logits [n_tok][n_expert] as bh_moe_route does (then selected and
 * weights must be NULL; selected_out / weights_out, if non-NULL, receive
 * it). A token's k experts must be distinct (else the device status
 * reports BH_EINVAL and out is not written). Every expert chosen by several
 * tokens is streamed once. One cooperative launch (all CTAs resident, grid
 * barriers between the gate|up, down and combine phases); scratch buffers
 * are owned by the context. */
int bh_q4k_moe(bh_ctx *ctx, const float *cur, int n_tok, const int32_t *selected, const float *weights,
               const float *router_logits, int norm_topk, const void *gate_exps, const void *up_exps,
               const void *down_exps, int n_expert, int n_embd, int n_ff, int k, float *out,
               int32_t *selected_out, float *weights_out, int fold, void *stream);

/* Expert-parallel share of bh_q4k_moe on one rank: only the pairs (token,
 * slot) routed to experts [expert_lo, expert_hi) are computed, from banks
 * holding exactly those experts (gate_own / up_own [expert_hi - expert_lo]
 * [n_ff][n_embd], down_own [..][n_embd][n_ff]) -- the sub-bank split that
 * BURN_MOE's pivot makes between its CPU and GPU banks (burn_moe_op.h:40-46).
 * dout [n_tok*k][n_embd] receives the unweighted expert output of every
 * owned pair and -0.0 in the rows of the others, so the element-wise sum of
 * dout over ranks owning disjoint ranges that cover all experts equals the
 * single-device expert outputs exactly; bh_moe_combine then forms out.
 * Routing as in bh_q4k_moe (every rank routes identically). */
int bh_q4k_moe_ep(bh_ctx *ctx, const float *cur, int n_tok, const int32_t *selected, const float *weights,
                  const float *router_logits, int norm_topk, const void *gate_own, const void *up_own,
                  const void *down_own, int n_expert, int expert_lo, int expert_hi, int n_embd, int n_ff, int k,
                  float *dout, int32_t *selected_out, float *weights_out, int fold, void *stream);

/* out[t][i] = (float) sum over slots s, in order, of (double)(dout[t*k+s][i] * weights[t][s])
 * (ggml_mul then ggml_sum_rows, forward.cpp:1099-1107); with residual != 0
 * the result is added to out instead. */
int bh_moe_combine(bh_ctx *ctx, const float *dout, const float *weights, int n_tok, int k, int n_embd, float *out,
                   int residual, void *stream);
/* bh_moe_combine over two expert-parallel shares computed on one device
 * (BURN_MOE's pivot split: bh_q4k_moe_ep on the experts [0, pivot) bank into
 * dout_a and on the [pivot, n_expert) bank into dout_b): each pair's row is
 * dout_a + dout_b, exact since one of them is -0.0. */
int bh_moe_combine_split(bh_ctx *ctx, const float *dout_a, const float *dout_b, const float *weights, int n_tok,
                         int k, int n_embd, float *out, int residual, void *stream);

/* The MoE layer stack of the 30B-A3B shape: per layer h += moe(RMSNorm(h) *
 * ffn_norm) with router logits seeded N(0, 1) per (layer, token), expert
 * banks seeded N(0, 0.02) and quantized to Q4_K on the device. One step runs
 * every layer for n_tok tokens, one cooperative launch per layer, captured
 * in a CUDA graph. */
typedef struct bh_moe_stack bh_moe_stack;
typedef struct bh_moe_config {
    int n_layer;   /* 48 */
    int n_embd;    /* 2048 */
    int n_ff;      /* 768 */
    int n_expert;  /* 128 */
    int k;         /* 8 */
    int n_tok;     /* tokens per step, 1..8 */
    float rms_eps; /* 1e-6 */
} bh_moe_config;

#define BH_MOE_GATE 0
#define BH_MOE_UP 1
#define BH_MOE_DOWN 2
#define BH_MOE_LOGITS 3    /* [n_tok][n_expert] fp32 */
#define BH_MOE_NORM 4      /* [n_embd] fp32 */
#define BH_MOE_SELECTED 5  /* [n_tok][k] int32, written by each step */
#define BH_MOE_WEIGHTS 6   /* [n_tok][k] fp32, written by each step */
#define BH_MOE_HIDDEN 7    /* [n_tok][n_embd] fp32 (layer == -1) */
#define BH_MOE_BARRIER 8   /* the layer kernels' grid-barrier words, 256 bytes (layer == -1) */

void bh_moe_default_config(bh_moe_config *cfg);
int bh_moe_stack_create(bh_ctx *ctx, const bh_moe_config *cfg, uint64_t seed, bh_moe_stack **out);
int bh_moe_stack_free(bh_moe_stack *st);
/* h [n_tok][n_embd] (device) is copied in, all layers run, the result is
 * written to h_out (device). Asynchronous on stream. */
int bh_moe_stack_step(bh_moe_stack *st, const float *h, float *h_out, void *stream);
/* The same step from and to host memory (copies inside the call). */
int bh_moe_stack_step_host(bh_moe_stack *st, const float *host_h, float *host_h_out);
/* Bytes of all expert weights, bytes of the experts the last step selected
 * (distinct experts per layer x bytes per expert, plus the activations the
 * matvecs read and write), and launches per step. */
int bh_moe_stack_info(bh_moe_stack *st, int64_t *weight_bytes, int64_t *step_bytes, int64_t *launches);
/* Device pointer and bytes of one tensor (ids above) of a layer. */
int bh_moe_stack_tensor(bh_moe_stack *st, int layer, int which, void **ptr, int64_t *bytes);

/* ------------------------------------------------------------------------
 * GGUF tensor reader -> device upload: the weights of a model file (the
 * reference engine's loader, desktop/engine/src/gguf_loader.cpp, binding
 * tensors in llama_weights.cpp:866-950). GGUF v2/v3 (vendor/ggml/include/
 * gguf.h); the file is memory-mapped read-only and every offset is checked
 * against its size (a truncated or corrupt file returns BH_EINVAL). Tensor
 * bytes are the GGML block rows the matvecs consume, uploaded unchanged.
 * ------------------------------------------------------------------------ */
typedef struct bh_gguf bh_gguf;
int bh_gguf_open(const char *path, bh_gguf **out);
int bh_gguf_close(bh_gguf *g);
int64_t bh_gguf_n_tensors(const bh_gguf *g);
int64_t bh_gguf_n_keys(const bh_gguf *g);
/* Index of a tensor / key by name, or -1. */
int64_t bh_gguf_find_tensor(const bh_gguf *g, const char *name);
int64_t bh_gguf_find_key(const bh_gguf *g, const char *key);
/* Name, ggml type id, dimensions, ne[4] (unused dims 1), byte offset in the
 * file and byte size (0 for a ggml type whose block size is not known here). */
int bh_gguf_tensor_info(const bh_gguf *g, int64_t i, const char **name, int *ggml_type, int *n_dims, int64_t *ne4,
                        uint64_t *file_offset, uint64_t *bytes);
/* The tensor's bytes in the mapping (host memory, valid until close). */
const void *bh_gguf_tensor_host(const bh_gguf *g, int64_t i);
/* Copy tensor i into device memory dst (dst_bytes >= its size) on stream;
 * returns once the copy has completed. */
int bh_gguf_upload(bh_ctx *ctx, const bh_gguf *g, int64_t i, void *dst, size_t dst_bytes, void *stream);
/* Key k's name and GGUF value type; its value as an integer (any integer or
 * bool type), a float (float or integer types) or a string (not
 * NUL-terminated; len bytes). */
int bh_gguf_key(const bh_gguf *g, int64_t k, const char **key, int *type);
int bh_gguf_get_int(const bh_gguf *g, int64_t k, int64_t *v);
int bh_gguf_get_float(const bh_gguf *g, int64_t k, double *v);
int bh_gguf_get_str(const bh_gguf *g, int64_t k, const char **s, uint64_t *len);

/* ggml_vec_dot_t-shaped shim (ggml-cpu.h:113) for the type_traits slot of
 * GGML_TYPE_Q4_K: one row of K = n values, HOST pointers vx (block_q4_K)
 * and vy (block_q8_K), nrc must be 1. Runs on device 0 through a
 * process-wide context, x86 fold. Slow (two copies per call); it exists so
 * the reference's row-level tests can drive the device path unchanged. */
void bh_ggml_vec_dot_q4_K_q8_K(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy,
                               size_t by, int nrc);

#ifdef __cplusplus
}
#endif
#endif /* BH_Q4K_H */
