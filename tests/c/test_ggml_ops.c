/* GPU check of the ggml graph nodes of shannon-prime-burnhard_b200/adapters
 * (built by that directory's Makefile against the reference's ggml headers,
 * run by tests/test_gpu_adapters.py).
 *
 * One ggml graph on the reference's own x86 CPU backend holds, over the same
 * tensors:
 *  - the stock routed-expert path of forward.cpp:1096-1107 (three
 *    ggml_mul_mat_id, ggml_silu, ggml_mul, the weighted sum over k through
 *    ggml_sum_rows) and bh_build_burn_moe_op with one bank and with the
 *    banks split at a pivot (views of the experts [0, pivot) and
 *    [pivot, n_expert));
 *  - ggml_mul_mat of a Q4_K weight and bh_ggml_mul_mat (the Q4_K branch of
 *    sp_crt_mul_mat), for column counts that are and are not multiples of 8.
 * Every node of ours must equal its stock counterpart bit for bit. Prints
 * "GGML OPS OK" and exits 0 on success. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "bh_ggml_ops.h"
#include "ggml-cpu.h"
#include "ggml.h"

static uint64_t rng_state = 0x9e3779b97f4a7c15ULL;

static double uniform(void) {
    /* splitmix64 */
    uint64_t z = (rng_state += 0x9e3779b97f4a7c15ULL);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    z ^= z >> 31;
    return ((double)(z >> 11) + 0.5) / 9007199254740992.0;
}

static float normal(float sd) {
    const double u1 = uniform(), u2 = uniform();
    return (float)(sd * sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

static struct ggml_tensor *q4k_tensor(struct ggml_context *g, int64_t k, int64_t rows, int64_t mats, float sd) {
    struct ggml_tensor *t = ggml_new_tensor_3d(g, GGML_TYPE_Q4_K, k, rows, mats);
    float *f = (float *)malloc(sizeof(float) * (size_t)(k * rows * mats));
    for (int64_t i = 0; i < k * rows * mats; ++i) f[i] = normal(sd);
    ggml_quantize_chunk(GGML_TYPE_Q4_K, f, t->data, 0, rows * mats, k, NULL);
    free(f);
    return t;
}

static int same_bits(const struct ggml_tensor *a, const struct ggml_tensor *b, const char *what) {
    const size_t n = (size_t)ggml_nelements(a);
    const uint32_t *x = (const uint32_t *)a->data, *y = (const uint32_t *)b->data;
    size_t bad = 0, first = 0;
    for (size_t i = 0; i < n; ++i)
        if (x[i] != y[i]) {
            if (!bad) first = i;
            ++bad;
        }
    if (bad) {
        float fx, fy;
        memcpy(&fx, &x[first], 4);
        memcpy(&fy, &y[first], 4);
        printf("FAIL %s: %zu of %zu values differ (first at %zu: %.9g vs %.9g)\n", what, bad, n, first, fx, fy);
        return 1;
    }
    printf("ok %s (%zu values)\n", what, n);
    return 0;
}

static int moe_case(bh_ctx *ctx, int n_embd, int n_ff, int n_expert, int k, int n_tok, int pivot) {
    struct ggml_init_params ip = {(size_t)512 << 20, NULL, false};
    struct ggml_context *g = ggml_init(ip);
    struct ggml_tensor *cur = ggml_new_tensor_2d(g, GGML_TYPE_F32, n_embd, n_tok);
    for (int i = 0; i < n_embd * n_tok; ++i) ((float *)cur->data)[i] = normal(1.0f);
    struct ggml_tensor *gate = q4k_tensor(g, n_embd, n_ff, n_expert, 0.02f);
    struct ggml_tensor *up = q4k_tensor(g, n_embd, n_ff, n_expert, 0.02f);
    struct ggml_tensor *down = q4k_tensor(g, n_ff, n_embd, n_expert, 0.02f);
    struct ggml_tensor *sel = ggml_new_tensor_2d(g, GGML_TYPE_I32, k, n_tok);
    struct ggml_tensor *wts = ggml_new_tensor_3d(g, GGML_TYPE_F32, 1, k, n_tok);
    for (int t = 0; t < n_tok; ++t) {
        /* k distinct experts per token, random order; weights positive */
        int used[256] = {0};
        for (int s = 0; s < k; ++s) {
            int e;
            do e = (int)(uniform() * n_expert); while (used[e]);
            used[e] = 1;
            ((int32_t *)sel->data)[t * k + s] = e;
            ((float *)wts->data)[t * k + s] = (float)(0.05 + uniform());
        }
    }
    /* the stock path (forward.cpp:1096-1107) */
    struct ggml_tensor *cur3 = ggml_reshape_3d(g, cur, n_embd, 1, n_tok);
    struct ggml_tensor *up_e = ggml_mul_mat_id(g, up, cur3, sel);
    struct ggml_tensor *gate_e = ggml_mul_mat_id(g, gate, cur3, sel);
    gate_e = ggml_silu(g, gate_e);
    struct ggml_tensor *par = ggml_mul(g, gate_e, up_e);
    struct ggml_tensor *down_e = ggml_mul_mat_id(g, down, par, sel);
    struct ggml_tensor *weighted = ggml_mul(g, down_e, wts);
    struct ggml_tensor *wk = ggml_cont(g, ggml_permute(g, weighted, 1, 0, 2, 3));
    struct ggml_tensor *stock = ggml_reshape_2d(g, ggml_sum_rows(g, wk), n_embd, n_tok);
    /* ours: one bank, and the banks split at the pivot */
    struct ggml_tensor *ours = bh_build_burn_moe_op(g, cur, sel, wts, gate, up, down, NULL, NULL, NULL, k, 0, ctx);
    struct ggml_tensor *lo[3], *hi[3], *bank[3] = {gate, up, down};
    for (int j = 0; j < 3; ++j) {
        struct ggml_tensor *b = bank[j];
        lo[j] = ggml_view_3d(g, b, b->ne[0], b->ne[1], pivot, b->nb[1], b->nb[2], 0);
        hi[j] = ggml_view_3d(g, b, b->ne[0], b->ne[1], n_expert - pivot, b->nb[1], b->nb[2], (size_t)pivot * b->nb[2]);
    }
    struct ggml_tensor *split =
        bh_build_burn_moe_op(g, cur, sel, wts, hi[0], hi[1], hi[2], lo[0], lo[1], lo[2], k, pivot, ctx);
    if (!ours || !split) {
        printf("FAIL bh_build_burn_moe_op returned NULL\n");
        return 1;
    }
    struct ggml_cgraph *gf = ggml_new_graph(g);
    ggml_build_forward_expand(gf, stock);
    ggml_build_forward_expand(gf, ours);
    ggml_build_forward_expand(gf, split);
    if (ggml_graph_compute_with_ctx(g, gf, 4) != GGML_STATUS_SUCCESS) {
        printf("FAIL graph compute\n");
        return 1;
    }
    int rc = bh_ggml_ops_last_error();
    if (rc) {
        printf("FAIL node error %d\n", rc);
        return 1;
    }
    char what[160];
    snprintf(what, sizeof what, "BURN_MOE %dx%d, %d experts, k %d, %d tokens", n_embd, n_ff, n_expert, k, n_tok);
    int bad = same_bits(stock, ours, what);
    snprintf(what, sizeof what, "BURN_MOE split at pivot %d, %d tokens", pivot, n_tok);
    bad |= same_bits(stock, split, what);
    ggml_free(g);
    return bad;
}

static int mul_mat_case(bh_ctx *ctx, int K, int M, int N) {
    struct ggml_init_params ip = {(size_t)256 << 20, NULL, false};
    struct ggml_context *g = ggml_init(ip);
    struct ggml_tensor *W = q4k_tensor(g, K, M, 1, 0.02f);
    W = ggml_reshape_2d(g, W, K, M);
    struct ggml_tensor *x = ggml_new_tensor_2d(g, GGML_TYPE_F32, K, N);
    for (int i = 0; i < K * N; ++i) ((float *)x->data)[i] = normal(1.0f);
    struct ggml_tensor *ref = ggml_mul_mat(g, W, x);
    struct ggml_tensor *ours = bh_ggml_mul_mat(g, W, x, ctx);
    struct ggml_cgraph *gf = ggml_new_graph(g);
    ggml_build_forward_expand(gf, ref);
    ggml_build_forward_expand(gf, ours);
    if (ggml_graph_compute_with_ctx(g, gf, 4) != GGML_STATUS_SUCCESS) {
        printf("FAIL graph compute\n");
        return 1;
    }
    int rc = bh_ggml_ops_last_error();
    if (rc) {
        printf("FAIL node error %d\n", rc);
        return 1;
    }
    char what[96];
    snprintf(what, sizeof what, "Q4_K mul_mat %dx%d x %d columns", M, K, N);
    int bad = same_bits(ref, ours, what);
    ggml_free(g);
    return bad;
}

int main(void) {
    bh_ctx *ctx = NULL;
    if (bh_init(0, &ctx) != BH_OK) {
        printf("FAIL bh_init\n");
        return 2;
    }
    int bad = 0;
    bad |= moe_case(ctx, 512, 256, 16, 4, 1, 6);
    bad |= moe_case(ctx, 512, 256, 16, 4, 3, 9);
    bad |= moe_case(ctx, 1024, 512, 32, 8, 11, 13);   /* two chunks of tokens */
    bad |= mul_mat_case(ctx, 1024, 777, 1);
    bad |= mul_mat_case(ctx, 2048, 1000, 8);
    bad |= mul_mat_case(ctx, 4096, 4096, 13);          /* two chunks of columns */
    const int cached = bh_ggml_ops_cached_weights();
    bh_ggml_ops_release();
    bh_free(ctx);
    if (!bad) printf("GGML OPS OK (%d weight tensors were uploaded once each)\n", cached);
    return bad;
}
