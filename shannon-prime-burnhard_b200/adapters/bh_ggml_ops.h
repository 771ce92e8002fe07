/* bh_ggml_ops.h — ggml graph nodes that run the reference engine's Q4_K hot
 * path on the B200 through include/bh_q4k.h.
 *
 * Two drop-ins for the reference engine's graph builders, compiled against
 * the engine's own ggml headers (vendor/ggml/include) and resolving the ggml
 * symbols from the engine process that loads them:
 *
 *  - bh_build_burn_moe_op: the BURN_MOE routed-expert node, the argument list
 *    of sp_build_burn_moe_op (desktop/engine/src/burn_moe_op.h:47-59) with
 *    the CRT dispatcher replaced by a bh_ctx: cur [n_embd, n_tokens] f32,
 *    selected [k, n_tokens] i32, weights [1, k, n_tokens] f32, the Q4_K
 *    expert banks holding experts [pivot, n_expert), and, when pivot > 0,
 *    the *_cpu banks holding experts [0, pivot). The node's value equals the
 *    stock path of forward.cpp:1096-1107 (three ggml_mul_mat_id, ggml_silu,
 *    ggml_mul, the weighted sum over k) on the x86 CPU backend, bit for bit.
 *  - bh_ggml_mul_mat: the Q4_K branch of sp_crt_mul_mat (forward.cpp:
 *    1266-1283): for a Q4_K weight W [K, M] and f32 x [K, N], a node [M, N]
 *    equal to ggml_mul_mat(W, x) on the x86 CPU backend bit for bit;
 *    other weight types fall through to ggml_mul_mat.
 *
 * Both nodes are ggml_custom_4d nodes (one task). Their callback reads the
 * inputs from host tensors (or with ggml_backend_tensor_get from backend
 * buffers), runs the device kernels on ctx's GPU and writes the result.
 * Weight tensors in host memory are uploaded to ctx's device on first use
 * and kept (keyed by device, data pointer and size) until
 * bh_ggml_ops_release; weights already in a CUDA buffer of ctx's device are
 * used in place. The nodes' user data is kept until bh_ggml_ops_release too
 * (after the graphs that hold them are done). The fold is BH_FOLD_X86, the
 * reference's path on x86 hosts. */
#ifndef BH_GGML_OPS_H
#define BH_GGML_OPS_H

#include "ggml.h"
#include "bh_q4k.h"

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_tensor *bh_build_burn_moe_op(struct ggml_context *gctx, struct ggml_tensor *cur,
                                         struct ggml_tensor *selected, struct ggml_tensor *weights,
                                         struct ggml_tensor *gate_exps, struct ggml_tensor *up_exps,
                                         struct ggml_tensor *down_exps, struct ggml_tensor *gate_exps_cpu,
                                         struct ggml_tensor *up_exps_cpu, struct ggml_tensor *down_exps_cpu,
                                         int n_expert_used, int pivot, bh_ctx *ctx);

struct ggml_tensor *bh_ggml_mul_mat(struct ggml_context *gctx, struct ggml_tensor *W, struct ggml_tensor *x,
                                    bh_ctx *ctx);

/* Errors met inside the callbacks since the last call (0: none): a BH_E*
 * code of the device call, or BH_EINVAL for an input the node cannot take
 * (the node's output is then left zero). Clears it. */
int bh_ggml_ops_last_error(void);

/* Device copies of host weight tensors kept by the nodes (for tests). */
int bh_ggml_ops_cached_weights(void);

/* Free every cached device copy of host weights and every node's user data
 * (no graph holding one of these nodes may be computed afterwards). */
void bh_ggml_ops_release(void);

#ifdef __cplusplus
}
#endif

#endif /* BH_GGML_OPS_H */
