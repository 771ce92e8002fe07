/*
 * ref_graph.c — the reference's own ggml CPU backend (vendored ggml 0.11.0,
 * compiled from the reference tree by oracle/Makefile into
 * oracle/_ref/libggml_graph.so) driven through ggml's public graph API.
 * TEST INFRASTRUCTURE AND CPU BASELINE ONLY: nothing of the product links it.
 *
 *  - rg_stack_*: the Qwen3-shaped decode step exactly as the reference engine
 *    builds it for one token (desktop/engine/src/forward.cpp:2663-2854
 *    build_block_decode: ggml_rms_norm * attn_norm, ggml_mul_mat for Wq / Wk /
 *    Wv, per-head ggml_rms_norm * q/k norm, ggml_rope_ext in NeoX mode,
 *    ggml_concat with the past K/V, ggml_repeat for GQA, ggml_mul_mat K.Q,
 *    ggml_scale 1/sqrt(head_dim), ggml_soft_max_ext, ggml_mul_mat V.softmax,
 *    Wo, ggml_add, ggml_rms_norm * ffn_norm, Wg / Wu, ggml_silu, ggml_mul,
 *    Wd, ggml_add; then forward.cpp:3410-3413 rms_norm * output_norm and the
 *    LM head ggml_mul_mat; the token is argmax() of engine.cpp:36-43).
 *    The graph is computed by ggml_graph_compute_with_ctx on the CPU
 *    backend's own thread pool, so every Q4_K matvec runs the stock path
 *    ggml_compute_forward_mul_mat (ggml-cpu.c:1241-1439): src1 quantized to
 *    Q8_K by from_float, then ggml_vec_dot_q4_K_q8_K in ggml's chunks.
 *    The KV cache is fp32 [n_ctx][n_head_kv][head_dim] per layer, as the
 *    engine's past_K / past_V graph inputs are (forward.cpp:3506); the new
 *    token's K (after RoPE) and V are written back at `pos` after the compute,
 *    as the engine's cache write-back does.
 *  - rg_mul_mat: one ggml_mul_mat node (Q4_K weight, f32 activations) at a
 *    given thread count, the "graph matmul" CPU legs.
 *  - rg_quantize_q4k / rg_fill_normal: host weight preparation for the CPU
 *    baseline (ggml_quantize_chunk -> quantize_row_q4_K_ref, over threads;
 *    the splitmix64 + Box-Muller generator the device stacks use).
 *
 * Tensor ids follow include/bh_q4k.h (BH_W_Q .. BH_T_V_CACHE).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "ggml.h"
#include "ggml-cpu.h"
#include "gguf.h"

enum { W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_PER_LAYER, W_OUTPUT = 7,
       T_ATTN_NORM = 8, T_FFN_NORM, T_Q_NORM, T_K_NORM, T_OUT_NORM, T_K_CACHE, T_V_CACHE };

typedef struct rg_config {
    int n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab, n_ctx;
    float rms_eps, rope_theta;
    int n_distinct; /* layers with their own weights; layer l uses the weights of l % n_distinct */
} rg_config;

typedef struct rg_layer {
    struct ggml_tensor *w[W_PER_LAYER];
    struct ggml_tensor *attn_norm, *ffn_norm, *q_norm, *k_norm;
} rg_layer;

typedef struct rg_stack {
    rg_config c;
    struct ggml_context *wctx; /* weights, norms, caches */
    rg_layer *layers;          /* n_distinct entries */
    struct ggml_tensor **kc, **vc; /* n_layer caches [head_dim, n_head_kv, n_ctx] */
    struct ggml_tensor *out_norm, *output;
    void *cbuf;                /* compute arena, reused by every call */
    size_t cbuf_bytes;
} rg_stack;

static size_t tensor_bytes(enum ggml_type t, int64_t ne0, int64_t ne1, int64_t ne2) {
    return ggml_row_size(t, ne0) * (size_t)ne1 * (size_t)ne2 + ggml_tensor_overhead() + 64;
}

void rg_stack_free(rg_stack *s) {
    if (!s) return;
    if (s->wctx) ggml_free(s->wctx);
    free(s->layers);
    free(s->kc);
    free(s->vc);
    free(s->cbuf);
    free(s);
}

rg_stack *rg_stack_create(const rg_config *cfg) {
    ggml_cpu_init();
    rg_stack *s = (rg_stack *)calloc(1, sizeof(rg_stack));
    if (!s) return NULL;
    s->c = *cfg;
    rg_config *c = &s->c;
    if (c->n_distinct < 1 || c->n_distinct > c->n_layer) c->n_distinct = c->n_layer;
    const int64_t qd = (int64_t)c->n_head * c->head_dim, kvd = (int64_t)c->n_head_kv * c->head_dim;
    const int64_t rows[W_PER_LAYER] = {qd, kvd, kvd, c->n_embd, c->n_ff, c->n_ff, c->n_embd};
    const int64_t cols[W_PER_LAYER] = {c->n_embd, c->n_embd, c->n_embd, qd, c->n_embd, c->n_embd, c->n_ff};
    size_t total = 1 << 20;
    for (int w = 0; w < W_PER_LAYER; ++w) total += (size_t)c->n_distinct * tensor_bytes(GGML_TYPE_Q4_K, cols[w], rows[w], 1);
    total += (size_t)c->n_distinct * (2 * tensor_bytes(GGML_TYPE_F32, c->n_embd, 1, 1) +
                                      2 * tensor_bytes(GGML_TYPE_F32, c->head_dim, 1, 1));
    total += (size_t)c->n_layer * 2 * tensor_bytes(GGML_TYPE_F32, c->head_dim, c->n_head_kv, c->n_ctx);
    total += tensor_bytes(GGML_TYPE_F32, c->n_embd, 1, 1) + tensor_bytes(GGML_TYPE_Q4_K, c->n_embd, c->n_vocab, 1);
    struct ggml_init_params ip = {total, NULL, false};
    s->wctx = ggml_init(ip);
    s->layers = (rg_layer *)calloc((size_t)c->n_distinct, sizeof(rg_layer));
    s->kc = (struct ggml_tensor **)calloc((size_t)c->n_layer, sizeof(void *));
    s->vc = (struct ggml_tensor **)calloc((size_t)c->n_layer, sizeof(void *));
    if (!s->wctx || !s->layers || !s->kc || !s->vc) { rg_stack_free(s); return NULL; }
    for (int l = 0; l < c->n_distinct; ++l) {
        rg_layer *L = &s->layers[l];
        for (int w = 0; w < W_PER_LAYER; ++w) L->w[w] = ggml_new_tensor_2d(s->wctx, GGML_TYPE_Q4_K, cols[w], rows[w]);
        L->attn_norm = ggml_new_tensor_1d(s->wctx, GGML_TYPE_F32, c->n_embd);
        L->ffn_norm = ggml_new_tensor_1d(s->wctx, GGML_TYPE_F32, c->n_embd);
        L->q_norm = ggml_new_tensor_1d(s->wctx, GGML_TYPE_F32, c->head_dim);
        L->k_norm = ggml_new_tensor_1d(s->wctx, GGML_TYPE_F32, c->head_dim);
    }
    for (int l = 0; l < c->n_layer; ++l) {
        s->kc[l] = ggml_new_tensor_3d(s->wctx, GGML_TYPE_F32, c->head_dim, c->n_head_kv, c->n_ctx);
        s->vc[l] = ggml_new_tensor_3d(s->wctx, GGML_TYPE_F32, c->head_dim, c->n_head_kv, c->n_ctx);
        memset(s->kc[l]->data, 0, ggml_nbytes(s->kc[l]));
        memset(s->vc[l]->data, 0, ggml_nbytes(s->vc[l]));
    }
    s->out_norm = ggml_new_tensor_1d(s->wctx, GGML_TYPE_F32, c->n_embd);
    s->output = ggml_new_tensor_2d(s->wctx, GGML_TYPE_Q4_K, c->n_embd, c->n_vocab);
    /* compute arena: every intermediate of one step (the GQA-repeated K/V of
     * each layer dominate) plus the logits and ggml's work buffer */
    const size_t per_layer = (size_t)8 * qd * c->n_ctx * 4 + (size_t)48 * (c->n_embd + c->n_ff + qd) * 4 +
                             (size_t)256 * ggml_tensor_overhead();
    s->cbuf_bytes = (size_t)c->n_layer * per_layer + (size_t)8 * c->n_vocab * 4 + ((size_t)64 << 20);
    s->cbuf = malloc(s->cbuf_bytes);
    if (!s->cbuf) { rg_stack_free(s); return NULL; }
    return s;
}

/* Host pointer and byte size of one tensor (the caller fills weights, norms
 * and caches). Weights: Q4_K rows of GGML layout. */
void *rg_stack_tensor(rg_stack *s, int layer, int which, size_t *bytes) {
    struct ggml_tensor *t = NULL;
    const rg_config *c = &s->c;
    if (which == W_OUTPUT && layer < 0) t = s->output;
    else if (which == T_OUT_NORM) t = s->out_norm;
    else if (which == T_K_CACHE || which == T_V_CACHE) {
        if (layer < 0 || layer >= c->n_layer) return NULL;
        t = which == T_K_CACHE ? s->kc[layer] : s->vc[layer];
    } else {
        if (layer < 0 || layer >= c->n_distinct) return NULL;
        rg_layer *L = &s->layers[layer];
        if (which >= 0 && which < W_PER_LAYER) t = L->w[which];
        else if (which == T_ATTN_NORM) t = L->attn_norm;
        else if (which == T_FFN_NORM) t = L->ffn_norm;
        else if (which == T_Q_NORM) t = L->q_norm;
        else if (which == T_K_NORM) t = L->k_norm;
    }
    if (!t) return NULL;
    if (bytes) *bytes = ggml_nbytes(t);
    return t->data;
}

/* One decode step at position pos (attention over 0..pos) from the
 * embedding x [n_embd]. Returns the token (first index of the maximum
 * logit), or -1 on failure. logits_out [n_vocab] and hidden_out [n_embd]
 * (the residual stream after the last layer) may be NULL. */
int rg_stack_decode(rg_stack *s, const float *x, int pos, int n_threads, float *logits_out, float *hidden_out) {
    const rg_config *c = &s->c;
    if (pos < 0 || pos >= c->n_ctx || n_threads < 1) return -1;
    const int hd = c->head_dim, nh = c->n_head, nkv = c->n_head_kv;
    const int64_t qd = (int64_t)nh * hd;
    struct ggml_init_params ip = {s->cbuf_bytes, s->cbuf, false};
    struct ggml_context *g = ggml_init(ip);
    if (!g) return -1;
    struct ggml_tensor *cur_x = ggml_new_tensor_2d(g, GGML_TYPE_F32, c->n_embd, 1);
    memcpy(cur_x->data, x, sizeof(float) * (size_t)c->n_embd);
    struct ggml_tensor *pos_t = ggml_new_tensor_1d(g, GGML_TYPE_I32, 1);
    ((int32_t *)pos_t->data)[0] = pos;
    struct ggml_tensor **kcap = (struct ggml_tensor **)calloc((size_t)c->n_layer, sizeof(void *));
    struct ggml_tensor **vcap = (struct ggml_tensor **)calloc((size_t)c->n_layer, sizeof(void *));
    if (!kcap || !vcap) { free(kcap); free(vcap); ggml_free(g); return -1; }
    struct ggml_tensor *xcur = cur_x;
    const float qk_scale = 1.0f / sqrtf((float)hd);
    for (int l = 0; l < c->n_layer; ++l) {
        const rg_layer *L = &s->layers[l % c->n_distinct];
        struct ggml_tensor *xa = ggml_rms_norm(g, xcur, c->rms_eps);
        xa = ggml_mul(g, xa, L->attn_norm);
        struct ggml_tensor *Q = ggml_mul_mat(g, L->w[W_Q], xa);
        struct ggml_tensor *K = ggml_mul_mat(g, L->w[W_K], xa);
        struct ggml_tensor *V = ggml_mul_mat(g, L->w[W_V], xa);
        Q = ggml_reshape_3d(g, Q, hd, nh, 1);
        K = ggml_reshape_3d(g, K, hd, nkv, 1);
        V = ggml_reshape_3d(g, V, hd, nkv, 1);
        Q = ggml_mul(g, ggml_rms_norm(g, Q, c->rms_eps), L->q_norm);
        K = ggml_mul(g, ggml_rms_norm(g, K, c->rms_eps), L->k_norm);
        Q = ggml_rope_ext(g, Q, pos_t, NULL, hd, GGML_ROPE_TYPE_NEOX, 0, c->rope_theta, 1.0f, 0.0f, 1.0f, 32.0f, 1.0f);
        K = ggml_rope_ext(g, K, pos_t, NULL, hd, GGML_ROPE_TYPE_NEOX, 0, c->rope_theta, 1.0f, 0.0f, 1.0f, 32.0f, 1.0f);
        V = ggml_cont(g, V);
        kcap[l] = K;
        vcap[l] = V;
        struct ggml_tensor *Kf = K, *Vf = V;
        if (pos > 0) {
            struct ggml_tensor *pk = ggml_view_3d(g, s->kc[l], hd, nkv, pos, s->kc[l]->nb[1], s->kc[l]->nb[2], 0);
            struct ggml_tensor *pv = ggml_view_3d(g, s->vc[l], hd, nkv, pos, s->vc[l]->nb[1], s->vc[l]->nb[2], 0);
            Kf = ggml_concat(g, pk, K, 2);
            Vf = ggml_concat(g, pv, V, 2);
        }
        const int kv_total = pos + 1;
        if (nh != nkv) {
            const int rep = nh / nkv;
            struct ggml_tensor *Kx = ggml_reshape_4d(g, Kf, hd, 1, nkv, kv_total);
            Kx = ggml_repeat(g, Kx, ggml_new_tensor_4d(g, GGML_TYPE_F32, hd, rep, nkv, kv_total));
            Kf = ggml_reshape_3d(g, Kx, hd, nh, kv_total);
            struct ggml_tensor *Vx = ggml_reshape_4d(g, Vf, hd, 1, nkv, kv_total);
            Vx = ggml_repeat(g, Vx, ggml_new_tensor_4d(g, GGML_TYPE_F32, hd, rep, nkv, kv_total));
            Vf = ggml_reshape_3d(g, Vx, hd, nh, kv_total);
        }
        struct ggml_tensor *Qp = ggml_cont(g, ggml_permute(g, Q, 0, 2, 1, 3));
        struct ggml_tensor *Kp = ggml_cont(g, ggml_permute(g, Kf, 0, 2, 1, 3));
        struct ggml_tensor *KQ = ggml_mul_mat(g, Kp, Qp);
        KQ = ggml_scale(g, KQ, qk_scale);
        KQ = ggml_soft_max_ext(g, KQ, NULL, 1.0f, 0.0f);
        struct ggml_tensor *Vp = ggml_cont(g, ggml_permute(g, Vf, 1, 2, 0, 3));
        struct ggml_tensor *attn = ggml_mul_mat(g, Vp, KQ);
        attn = ggml_cont(g, ggml_permute(g, attn, 0, 2, 1, 3));
        attn = ggml_reshape_2d(g, attn, qd, 1);
        xcur = ggml_add(g, xcur, ggml_mul_mat(g, L->w[W_O], attn));
        struct ggml_tensor *xb = ggml_mul(g, ggml_rms_norm(g, xcur, c->rms_eps), L->ffn_norm);
        struct ggml_tensor *gate = ggml_mul_mat(g, L->w[W_GATE], xb);
        struct ggml_tensor *up = ggml_mul_mat(g, L->w[W_UP], xb);
        struct ggml_tensor *ffn = ggml_mul(g, ggml_silu(g, gate), up);
        xcur = ggml_add(g, xcur, ggml_mul_mat(g, L->w[W_DOWN], ffn));
    }
    struct ggml_tensor *hfin = xcur;
    struct ggml_tensor *h = ggml_mul(g, ggml_rms_norm(g, hfin, c->rms_eps), s->out_norm);
    struct ggml_tensor *logits = ggml_mul_mat(g, s->output, h);
    struct ggml_cgraph *gf = ggml_new_graph_custom(g, 16 * GGML_DEFAULT_GRAPH_SIZE, false);
    ggml_build_forward_expand(gf, logits);
    for (int l = 0; l < c->n_layer; ++l) {
        ggml_build_forward_expand(gf, kcap[l]);
        ggml_build_forward_expand(gf, vcap[l]);
    }
    const enum ggml_status st = ggml_graph_compute_with_ctx(g, gf, n_threads);
    int tok = -1;
    if (st == GGML_STATUS_SUCCESS) {
        /* the cache write-back of the new token's K and V at pos */
        const size_t row = sizeof(float) * (size_t)hd * nkv;
        for (int l = 0; l < c->n_layer; ++l) {
            memcpy((char *)s->kc[l]->data + (size_t)pos * row, kcap[l]->data, row);
            memcpy((char *)s->vc[l]->data + (size_t)pos * row, vcap[l]->data, row);
        }
        const float *lg = (const float *)logits->data;
        /* engine.cpp:36-43: first index of the strict maximum */
        int best = 0;
        float bv = lg[0];
        for (int i = 1; i < c->n_vocab; ++i)
            if (lg[i] > bv) { bv = lg[i]; best = i; }
        tok = best;
        if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)c->n_vocab);
        if (hidden_out) memcpy(hidden_out, hfin->data, sizeof(float) * (size_t)c->n_embd);
    }
    free(kcap);
    free(vcap);
    ggml_free(g);
    return tok;
}

/* y [b][n] = W [n rows of k] . x [b][k] through one ggml_mul_mat node. */
int rg_mul_mat(const void *w, int64_t n, int64_t k, const float *x, int b, float *y, int n_threads) {
    ggml_cpu_init();
    const size_t need = tensor_bytes(GGML_TYPE_F32, k, b, 1) + tensor_bytes(GGML_TYPE_F32, n, b, 1) +
                        tensor_bytes(GGML_TYPE_Q8_K, k, b, 1) * (size_t)(n_threads + 1) + 4 * ggml_tensor_overhead() +
                        ggml_graph_overhead() + ((size_t)16 << 20);
    struct ggml_init_params ip = {need, NULL, false};
    struct ggml_context *g = ggml_init(ip);
    if (!g) return -1;
    /* the weight tensor points at the caller's bytes (no copy) */
    struct ggml_tensor *wt = ggml_new_tensor_2d(g, GGML_TYPE_Q4_K, k, n);
    wt->data = (void *)w;
    struct ggml_tensor *xt = ggml_new_tensor_2d(g, GGML_TYPE_F32, k, b);
    memcpy(xt->data, x, sizeof(float) * (size_t)k * b);
    struct ggml_tensor *yt = ggml_mul_mat(g, wt, xt);
    struct ggml_cgraph *gf = ggml_new_graph(g);
    ggml_build_forward_expand(gf, yt);
    const enum ggml_status st = ggml_graph_compute_with_ctx(g, gf, n_threads);
    if (st == GGML_STATUS_SUCCESS) memcpy(y, yt->data, sizeof(float) * (size_t)n * b);
    ggml_free(g);
    return st == GGML_STATUS_SUCCESS ? 0 : -1;
}

/* ---------------------------------------------------------------- host prep */
typedef struct prep_job {
    const float *src;
    float *fdst;
    void *qdst;
    int64_t r0, r1, k;
    uint64_t seed;
    double mean, std;
} prep_job;

static void *quantize_rows(void *arg) {
    const prep_job *j = (const prep_job *)arg;
    if (j->r1 > j->r0)
        ggml_quantize_chunk(GGML_TYPE_Q4_K, j->src, j->qdst, j->r0 * j->k, j->r1 - j->r0, j->k, NULL);
    return NULL;
}

/* rows x k fp32 -> Q4_K (ggml_quantize_chunk -> quantize_row_q4_K_ref), rows
 * split over n_threads threads. */
int rg_quantize_q4k(const float *src, void *dst, int64_t rows, int64_t k, int n_threads) {
    ggml_cpu_init();
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    prep_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].src = src;
        jobs[t].qdst = dst;
        jobs[t].k = k;
        jobs[t].r0 = rows * t / n_threads;
        jobs[t].r1 = rows * (t + 1) / n_threads;
        pthread_create(&th[t], NULL, quantize_rows, &jobs[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* splitmix64 -> two 53-bit uniforms -> Box-Muller in double: element e of
 * the stream (seed) is mean + std * z(e), the generator of the device
 * stacks' fill_normal and of the oracle. */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
static inline double unit53(uint64_t seed, uint64_t ctr) {
    return (double)(mix64(seed + (ctr + 1u) * 0x9e3779b97f4a7c15ULL) >> 11) * 0x1.0p-53;
}

static void *fill_rows(void *arg) {
    const prep_job *j = (const prep_job *)arg;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t e = j->r0; e < j->r1; ++e) {
        const int64_t pair = e >> 1;
        const double u1 = 1.0 - unit53(j->seed, (uint64_t)(2 * pair));
        const double u2 = unit53(j->seed, (uint64_t)(2 * pair + 1));
        const double r = sqrt(-2.0 * log(u1));
        const double z = (e & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        j->fdst[e - j->k] = (float)(j->mean + j->std * z);
    }
    return NULL;
}

/* out[i] = mean + std * z(first + i), i < n, over n_threads threads. */
int rg_fill_normal(float *out, int64_t n, int64_t first, uint64_t seed, double mean, double std, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    prep_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].fdst = out;
        jobs[t].k = first; /* element index of out[0] */
        jobs[t].r0 = first + n * t / n_threads;
        jobs[t].r1 = first + n * (t + 1) / n_threads;
        jobs[t].seed = seed;
        jobs[t].mean = mean;
        jobs[t].std = std;
        pthread_create(&th[t], NULL, fill_rows, &jobs[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* The build's thread count default and the CPU branch ggml uses. */
int rg_has_avx2(void) { return ggml_cpu_has_avx2() && ggml_cpu_has_fma() && ggml_cpu_has_f16c(); }

/* The direct row loop (no graph): y[r] = vec_dot(W row r, xq) for every row,
 * one thread, through the CPU backend's own type-traits entry for Q4_K
 * (ggml_vec_dot_q4_K_q8_K, arch/x86/quants.c:1900 on AVX2 hosts); xq is the
 * Q8_K activation from the backend's own from_float (quantize_row_q8_K). */
int rg_vec_dot_rows_type(int type, const void *w, int64_t n, int64_t k, const float *x, float *y) {
    ggml_cpu_init();
    if (type != GGML_TYPE_Q4_K && type != GGML_TYPE_Q6_K) return -1;
    const struct ggml_type_traits_cpu *tq = ggml_get_type_traits_cpu((enum ggml_type)type);
    const struct ggml_type_traits_cpu *t8 = ggml_get_type_traits_cpu(GGML_TYPE_Q8_K);
    if (!tq || !tq->vec_dot || !t8 || !t8->from_float) return -1;
    const size_t rb = ggml_row_size((enum ggml_type)type, k);
    void *xq = malloc(ggml_row_size(GGML_TYPE_Q8_K, k));
    if (!xq) return -1;
    t8->from_float(x, xq, k);
    for (int64_t r = 0; r < n; ++r) tq->vec_dot((int)k, y + r, 0, (const char *)w + (size_t)r * rb, 0, xq, 0, 1);
    free(xq);
    return 0;
}

int rg_vec_dot_rows(const void *w, int64_t n, int64_t k, const float *x, float *y) {
    return rg_vec_dot_rows_type(GGML_TYPE_Q4_K, w, n, k, x, y);
}

/* rows x k fp32 -> Q6_K (ggml_quantize_chunk -> quantize_row_q6_K_ref), one thread */
int rg_quantize_q6k(const float *src, void *dst, int64_t rows, int64_t k) {
    ggml_cpu_init();
    ggml_quantize_chunk(GGML_TYPE_Q6_K, src, dst, 0, rows, k, NULL);
    return 0;
}


/* A GGUF file written by the reference's own gguf writer (gguf.cpp): n 2-D
 * tensors (names, ggml types, ne0 x ne1, host bytes), u32 key/values, one
 * string key/value and one f32 key/value. Test fixture writer only. */
int rg_gguf_write(const char *path, int n, const char **names, const int *types, const int64_t *ne0,
                  const int64_t *ne1, const void **data, int n_u32, const char **u32_keys, const uint32_t *u32_vals,
                  const char *str_key, const char *str_val, const char *f32_key, float f32_val) {
    struct ggml_init_params ip = {(size_t)(n + 1) * ggml_tensor_overhead() + 4096, NULL, true};
    struct ggml_context *g = ggml_init(ip);
    if (!g) return -1;
    struct gguf_context *gg = gguf_init_empty();
    for (int i = 0; i < n_u32; ++i) gguf_set_val_u32(gg, u32_keys[i], u32_vals[i]);
    if (str_key) gguf_set_val_str(gg, str_key, str_val);
    if (f32_key) gguf_set_val_f32(gg, f32_key, f32_val);
    for (int i = 0; i < n; ++i) {
        struct ggml_tensor *t = ggml_new_tensor_2d(g, (enum ggml_type)types[i], ne0[i], ne1[i]);
        ggml_set_name(t, names[i]);
        t->data = (void *)data[i];
        gguf_add_tensor(gg, t);
    }
    const bool ok = gguf_write_to_file(gg, path, false);
    gguf_free(gg);
    ggml_free(g);
    return ok ? 0 : -1;
}