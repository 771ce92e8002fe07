/*
 * ref_driver.c — entry points into the reference's own Q4_K / Q8_K code,
 * compiled from the reference tree into oracle/_ref/libq4k_ref.so.
 * TEST INFRASTRUCTURE ONLY: pins the oracle restatement, generates the
 * golden fixtures, and is the timed CPU baseline (--impl reference).
 *
 * The functions called here are the reference's, unmodified:
 *   quantize_row_q4_K_ref        ggml-quants.c:1395
 *   quantize_row_q8_K_ref        ggml-quants.c:2692
 *   quantize_row_q8_K (x86)      ggml-cpu/arch/x86/quants.c:505
 *   dequantize_row_q4_K          ggml-quants.c:1467
 *   ggml_vec_dot_q4_K_q8_K_generic  ggml-cpu/quants.c:645
 *   ggml_vec_dot_q4_K_q8_K (AVX2)   ggml-cpu/arch/x86/quants.c:1900
 *
 * ref_mul_mat() drives them the way ggml_compute_forward_mul_mat does
 * (ggml-cpu/ggml-cpu.c:1241-1439): every thread quantizes its K-slice of
 * each activation column to Q8_K with the type's from_float, a barrier,
 * then output rows are handed out in chunks (64 rows when one operand is a
 * vector, 16 otherwise; re-chunked per thread when there are fewer than
 * 4 chunks per thread), each row computed by vec_dot.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void quantize_row_q4_K_ref(const float *x, void *y, int64_t k);
void quantize_row_q8_K_ref(const float *x, void *y, int64_t k);
void quantize_row_q8_K(const float *x, void *y, int64_t k);
void dequantize_row_q4_K(const void *x, float *y, int64_t k);
void ggml_vec_dot_q4_K_q8_K_generic(int n, float *s, size_t bs, const void *vx, size_t bx,
                                    const void *vy, size_t by, int nrc);
void ggml_vec_dot_q4_K_q8_K(int n, float *s, size_t bs, const void *vx, size_t bx,
                            const void *vy, size_t by, int nrc);

int ref_has_avx2(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
           __builtin_cpu_supports("f16c");
}

void ref_quantize_row_q4k(const float *x, void *y, int64_t k) { quantize_row_q4_K_ref(x, y, k); }
void ref_quantize_row_q8k_ref(const float *x, void *y, int64_t k) { quantize_row_q8_K_ref(x, y, k); }
void ref_quantize_row_q8k(const float *x, void *y, int64_t k) { quantize_row_q8_K(x, y, k); }
void ref_dequantize_row_q4k(const void *x, float *y, int64_t k) { dequantize_row_q4_K(x, y, k); }

float ref_vec_dot_generic(int n, const void *w, const void *x) {
    float s = 0;
    ggml_vec_dot_q4_K_q8_K_generic(n, &s, 0, w, 0, x, 0, 1);
    return s;
}
float ref_vec_dot_x86(int n, const void *w, const void *x) {
    float s = 0;
    ggml_vec_dot_q4_K_q8_K(n, &s, 0, w, 0, x, 0, 1);
    return s;
}

/* ---------------- thread pool ---------------- */

typedef struct ref_pool ref_pool;
typedef void (*ref_task)(ref_pool *p, int ith);

struct ref_pool {
    int nth;
    pthread_t *th;
    pthread_mutex_t mu;
    pthread_cond_t cv_go, cv_done;
    uint64_t gen;
    int pending, quit;
    ref_task task;
    pthread_barrier_t bar;
    atomic_long next_chunk;
    /* current mul_mat arguments */
    const uint8_t *W;
    const float *X;
    uint8_t *Xq;
    float *Y;
    int64_t N, K;
    int B;
};

typedef struct { ref_pool *p; int ith; } ref_worker_arg;

static void *ref_worker(void *a) {
    ref_worker_arg *wa = (ref_worker_arg *)a;
    ref_pool *p = wa->p;
    const int ith = wa->ith;
    free(wa);
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (p->gen == seen && !p->quit) pthread_cond_wait(&p->cv_go, &p->mu);
        if (p->quit) { pthread_mutex_unlock(&p->mu); return NULL; }
        seen = p->gen;
        ref_task t = p->task;
        pthread_mutex_unlock(&p->mu);
        t(p, ith);
        pthread_mutex_lock(&p->mu);
        if (--p->pending == 0) pthread_cond_signal(&p->cv_done);
        pthread_mutex_unlock(&p->mu);
    }
}

void *ref_pool_create(int nth) {
    if (nth < 1) nth = 1;
    ref_pool *p = (ref_pool *)calloc(1, sizeof(ref_pool));
    p->nth = nth;
    p->th = (pthread_t *)calloc((size_t)nth, sizeof(pthread_t));
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_go, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    pthread_barrier_init(&p->bar, NULL, (unsigned)nth);
    for (int t = 1; t < nth; ++t) {
        ref_worker_arg *wa = (ref_worker_arg *)malloc(sizeof(*wa));
        wa->p = p;
        wa->ith = t;
        pthread_create(&p->th[t], NULL, ref_worker, wa);
    }
    return p;
}

void ref_pool_free(void *vp) {
    ref_pool *p = (ref_pool *)vp;
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->quit = 1;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    for (int t = 1; t < p->nth; ++t) pthread_join(p->th[t], NULL);
    pthread_barrier_destroy(&p->bar);
    free(p->th);
    free(p);
}

static void pool_run(ref_pool *p, ref_task t) {
    pthread_mutex_lock(&p->mu);
    p->task = t;
    p->pending = p->nth - 1;
    p->gen++;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    t(p, 0);
    pthread_mutex_lock(&p->mu);
    while (p->pending > 0) pthread_cond_wait(&p->cv_done, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

static void mul_mat_task(ref_pool *p, int ith) {
    const int nth = p->nth;
    const int64_t nb = p->K / 256;
    const int64_t xrow = nb * 292, wrow = nb * 144;
    /* from_float on this thread's slice of blocks of every column */
    const int64_t b0 = ith * nb / nth, b1 = (ith + 1) * nb / nth;
    for (int c = 0; c < p->B; ++c)
        if (b1 > b0)
            quantize_row_q8_K(p->X + c * p->K + b0 * 256, p->Xq + c * xrow + b0 * 292, (b1 - b0) * 256);
    if (ith == 0) atomic_store(&p->next_chunk, nth);
    pthread_barrier_wait(&p->bar);

    const int64_t nr0 = p->N, nr1 = p->B;
    int64_t chunk = (nr0 == 1 || nr1 == 1) ? 64 : 16;
    int64_t nc0 = (nr0 + chunk - 1) / chunk, nc1 = (nr1 + chunk - 1) / chunk;
    if (nc0 * nc1 < (int64_t)nth * 4) {
        nc0 = nr0 > nr1 ? nth : 1;
        nc1 = nr0 > nr1 ? 1 : nth;
    }
    const int64_t dr0 = (nr0 + nc0 - 1) / nc0, dr1 = (nr1 + nc1 - 1) / nc1;
    long cur = ith;
    while (cur < nc0 * nc1) {
        const int64_t i0 = cur % nc0, i1 = cur / nc0;
        const int64_t r0s = dr0 * i0, r0e = r0s + dr0 < nr0 ? r0s + dr0 : nr0;
        const int64_t r1s = dr1 * i1, r1e = r1s + dr1 < nr1 ? r1s + dr1 : nr1;
        for (int64_t c = r1s; c < r1e; ++c)
            for (int64_t r = r0s; r < r0e; ++r)
                ggml_vec_dot_q4_K_q8_K((int)p->K, p->Y + c * p->N + r, 0, p->W + r * wrow, 0,
                                       p->Xq + c * xrow, 0, 1);
        if (nth >= nc0 * nc1) break;
        cur = atomic_fetch_add(&p->next_chunk, 1);
    }
}

/* Y[c*N + r] = W[r] . q8k(X[c]);  X fp32 [B][K]; xq_scratch >= B*K/256*292 bytes */
void ref_mul_mat(void *vp, const void *W, int64_t N, int64_t K, const float *X, int B,
                 void *xq_scratch, float *Y) {
    ref_pool *p = (ref_pool *)vp;
    p->W = (const uint8_t *)W;
    p->X = X;
    p->Xq = (uint8_t *)xq_scratch;
    p->Y = Y;
    p->N = N;
    p->K = K;
    p->B = B;
    pool_run(p, mul_mat_task);
}

int ref_pool_threads(void *vp) { return ((ref_pool *)vp)->nth; }

/* ---- the expert glue through the reference's own vec.cpp ---------------- */
typedef double ggml_float;
ggml_float ggml_vec_soft_max_f32(const int n, float *y, const float *x, float max);
void ggml_vec_silu_f32(const int n, float *y, const float *x);

/* One row of ggml_compute_forward_soft_max_f32 (ggml-cpu/ops.cpp:5365-5382)
 * with scale 1 and no mask or sinks. */
void ref_soft_max(const float *x, int n, float *y) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) mx = x[i] > mx ? x[i] : mx;   /* ggml_vec_max_f32 */
    ggml_float sum = ggml_vec_soft_max_f32(n, y, x, mx);
    sum = 1.0 / sum;
    const float v = (float)sum;                                /* ggml_vec_scale_f32's float argument */
    for (int i = 0; i < n; ++i) y[i] *= v;
}

void ref_silu(const float *x, int n, float *y) { ggml_vec_silu_f32(n, y, x); }

/* exp through the reference's own SIMD kernel: ggml_vec_soft_max_f32 with
 * max 0 stores ggml_v_expf(x - 0) = ggml_v_expf(x) for every group of 8
 * (n % 8 tail elements go through libm expf). */
void ref_vexpf(const float *x, int n, float *y) { (void)ggml_vec_soft_max_f32(n, y, x, 0.0f); }
