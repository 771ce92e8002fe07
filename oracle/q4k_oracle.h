/*
 * q4k_oracle.h — CPU restatement of the reference's Q4_K x Q8_K arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the
 * sm_100a kernels; it is never linked into, loaded by, or called from the
 * product path. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may use it.
 *
 * Parity pinned: q4k_oracle.c is checked byte-for-byte / bit-for-bit
 * against the reference's own ggml sources compiled into oracle/_ref
 * (see oracle/Makefile) and against the committed fixtures in
 * tests/golden/ that were produced by that compiled reference.
 *
 * Block layouts (vendor/ggml/src/ggml-common.h:317-328, 360-366):
 *   block_q4_K : 144 B / 256 weights = fp16 d | fp16 dmin | u8 scales[12] | u8 qs[128]
 *   block_q8_K : 292 B / 256 values  = f32 d  | i8 qs[256] | i16 bsums[16]
 */
#ifndef BH_Q4K_ORACLE_H
#define BH_Q4K_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BHO_QK 256
#define BHO_Q4K_BYTES 144
#define BHO_Q8K_BYTES 292

/* fold selectors for the fp32 reduction order */
#define BHO_FOLD_X86     0  /* ggml-cpu/arch/x86/quants.c:1900-1983 (AVX2 branch) */
#define BHO_FOLD_GENERIC 1  /* ggml-cpu/quants.c:645-718 */

float    bho_fp16_to_fp32(uint16_t h);
uint16_t bho_fp32_to_fp16(float f);

/* Counter-based normal generator: splitmix64 -> two 53-bit uniforms ->
 * Box-Muller in double -> rounded to float. Element e of the stream is a
 * pure function of (seed, e), so any sub-range can be regenerated. */
void bho_fill_normal(float *out, int64_t n, uint64_t seed, double mean, double stddev);
void bho_fill_normal_range(float *out, int64_t first, int64_t n, uint64_t seed,
                           double mean, double stddev);

/* quantize_row_q4_K_ref (ggml-quants.c:1395-1465), k % 256 == 0 */
void bho_quantize_row_q4k(const float *x, void *y, int64_t k);
/* rows of n_per_row each, nthreads >= 1 (rows are independent) */
void bho_quantize_q4k(const float *x, void *y, int64_t nrow, int64_t n_per_row, int nthreads);
/* dequantize_row_q4_K (ggml-quants.c:1467-1489) */
void bho_dequantize_row_q4k(const void *x, float *y, int64_t k);
/* quantize_row_q8_K_ref (ggml-quants.c:2692-2729); all-zero blocks get bsums = 0 */
void bho_quantize_row_q8k(const float *x, void *y, int64_t k);

/* one row . one column */
float bho_vec_dot_generic(int n, const void *w_row, const void *x_q8k);
float bho_vec_dot_x86(int n, const void *w_row, const void *x_q8k);

/* Y[b*N + r] = W[r] . X[b]   (GGML dst [N, B], column b contiguous) */
/* Q6_K (210-byte blocks) x Q8_K, the x86 AVX2 fold of ggml_vec_dot_q6_K_q8_K */
#define BHO_Q6K_BYTES 210
float bho_vec_dot_q6k_x86(int n, const void *vw, const void *vx);
void bho_matvec_q6k(const void *W, int64_t N, int64_t K, const void *Xq, int B, float *Y, int nthreads);
void bho_matvec(const void *W, int64_t N, int64_t K, const void *Xq, int B,
                float *Y, int fold, int nthreads);

/* Exact integer partials, layout [B][N][nb][9] int32:
 *   [..][j] (j < 8) = sum_{t<32} q4[256i+32j+t] * q8[256i+32j+t]  (unscaled)
 *   [..][8]        = sum_{j<8} min6_j * (bsums[2j] + bsums[2j+1])  (the min term) */
void bho_partials(const void *W, int64_t N, int64_t K, const void *Xq, int B, int32_t *out);

/* engine.cpp:36-43: first index of the strict maximum */
int64_t bho_argmax(const float *v, int64_t n);

/* ---- routed-expert FFN glue (forward.cpp:1001-1118), see q4k_oracle.c ---- */
float bho_expf(float x);   /* one lane of ggml's AVX2 ggml_v_expf; identical to the GPU's */
float bho_silu(float x);   /* x / (1 + exp(-x)) */
void  bho_expf_n(const float *x, int64_t n, float *y);
void  bho_silu_n(const float *x, int64_t n, float *y);
void  bho_rmsnorm(const float *x, const float *gamma, int n, float eps, float *y);
/* softmax -> top-k (slots 0/1 swapped) -> gather -> renormalise; n_expert <= 1024 */
void  bho_moe_route(const float *logits, int n_expert, int k, int norm, int32_t *ids, float *w);
void  bho_moe_ffn(const float *cur, int T, const int32_t *ids, const float *w, int k,
                  const void *gate, const void *up, const void *down, int n_embd, int n_ff,
                  float *out, float *gu_opt, float *dout_opt, int fold, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
