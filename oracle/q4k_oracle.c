/*
 * q4k_oracle.c — CPU restatement of the reference's Q4_K x Q8_K arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; never on the product path).
 * Must be compiled with -ffp-contract=off: every float operation below is a
 * separately rounded IEEE binary32 operation, exactly as the C source of the
 * reference reads; the only fused multiply-adds are the explicit ones the
 * reference's AVX2 branch issues (_mm256_fmadd_ps / _mm_fmadd_ps), which are
 * written here as fmaf().
 *
 * Every function cites the reference lines it restates (paths are relative
 * to vendor/ggml/src/ in the reference tree).
 */
#include "q4k_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* small helpers                                                       */
/* ------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline int16_t rds16(const uint8_t *p) { int16_t v; memcpy(&v, p, 2); return v; }
static inline float rdf32(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

/* IEEE binary16 -> binary32, exact (ggml-impl.h:384-405 computes the same
 * value; the CPU backend uses F16C _cvtsh_ss on x86, also exact). */
float bho_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    if (ex == 0) {
        /* zero or subnormal: man * 2^-24, exact in binary32 */
        const float mag = (float)man * 5.9604644775390625e-08f;
        return u2f(f2u(mag) | sign);
    }
    if (ex == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((ex + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16, round to nearest even (the value ggml-impl.h:407-431
 * produces for every finite input; NaN maps to 0x7e00 | sign as there). */
uint16_t bho_fp32_to_fp16(float f) {
    const uint32_t x = f2u(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return sign | 0x7e00u;
    if (ax >= 0x477ff000u) return sign | 0x7c00u; /* |f| >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                       /* below 2^-14: fp16 subnormal */
        const uint32_t e = ax >> 23;
        const uint32_t shift = 126u - e;          /* value * 2^24 = M >> shift */
        if (shift >= 32u) return sign;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return sign | (uint16_t)q;
    }
    uint32_t h = ((ax >> 23) - 112u) << 10 | ((ax & 0x7fffffu) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

/* ggml-quants.c:559-563: round-half-even via the 1.5*2^23 bias */
static inline int round_biased(float v) {
    const float b = v + 12582912.f;
    return (int)(f2u(b) & 0x007fffffu) - 0x00400000;
}

/* ------------------------------------------------------------------ */
/* seeded inputs                                                       */
/* ------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
static inline double unit53(uint64_t seed, uint64_t ctr) {
    const uint64_t z = mix64(seed + (ctr + 1u) * 0x9e3779b97f4a7c15ULL);
    return (double)(z >> 11) * 0x1.0p-53;
}

void bho_fill_normal_range(float *out, int64_t first, int64_t n, uint64_t seed,
                           double mean, double stddev) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t t = 0; t < n; ++t) {
        const int64_t e = first + t;
        const int64_t pair = e >> 1;
        const double u1 = 1.0 - unit53(seed, (uint64_t)(2 * pair));   /* (0, 1] */
        const double u2 = unit53(seed, (uint64_t)(2 * pair + 1));
        const double r = sqrt(-2.0 * log(u1));
        const double z = (e & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[t] = (float)(mean + stddev * z);
    }
}

void bho_fill_normal(float *out, int64_t n, uint64_t seed, double mean, double stddev) {
    bho_fill_normal_range(out, 0, n, seed, mean, stddev);
}

/* ------------------------------------------------------------------ */
/* Q4_K quantizer                                                      */
/* ------------------------------------------------------------------ */

/* Weighted asymmetric 4-bit fit of one 32-value sub-block with a grid
 * search over the inverse scale: ggml-quants.c:737-816 (make_qkx2_quants)
 * with nmax = 15, rmin = -1, rdelta = 0.1, nstep = 20, squared error.
 * Returns the scale; *neg_min receives -min (>= 0). */
static float fit_subblock(const float *x, const float *w, uint8_t *L, float *neg_min) {
    const int n = 32, nmax = 15, nstep = 20;
    const float rmin = -1.f, rdelta = 0.1f;
    uint8_t trial[32];

    float lo = x[0], hi = x[0];
    float sw = w[0];
    float sx = sw * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
        sw += w[i];
        sx += w[i] * x[i];
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
        memset(L, 0, (size_t)n);
        *neg_min = -lo;
        return 0.f;
    }
    float inv = nmax / (hi - lo);
    float scale = 1 / inv;
    float best = 0;
    for (int i = 0; i < n; ++i) {
        int l = round_biased(inv * (x[i] - lo));
        l = l < 0 ? 0 : (l > nmax ? nmax : l);
        L[i] = (uint8_t)l;
        float diff = scale * L[i] + lo - x[i];
        diff = diff * diff;
        best += w[i] * diff;
    }
    for (int is = 0; is <= nstep; ++is) {
        inv = (rmin + rdelta * is + nmax) / (hi - lo);
        float s_l = 0, s_l2 = 0, s_xl = 0;
        for (int i = 0; i < n; ++i) {
            int l = round_biased(inv * (x[i] - lo));
            l = l < 0 ? 0 : (l > nmax ? nmax : l);
            trial[i] = (uint8_t)l;
            s_l += w[i] * l;
            s_l2 += w[i] * l * l;
            s_xl += w[i] * l * x[i];
        }
        const float D = sw * s_l2 - s_l * s_l;
        if (D > 0) {
            float t_scale = (sw * s_xl - sx * s_l) / D;
            float t_min = (s_l2 * sx - s_l * s_xl) / D;
            if (t_min > 0) {
                t_min = 0;
                t_scale = s_xl / s_l2;
            }
            float err = 0;
            for (int i = 0; i < n; ++i) {
                float diff = t_scale * trial[i] + t_min - x[i];
                diff = diff * diff;
                err += w[i] * diff;
            }
            if (err < best) {
                memcpy(L, trial, (size_t)n);
                best = err;
                scale = t_scale;
                lo = t_min;
            }
        }
    }
    *neg_min = -lo;
    return scale;
}

/* 6-bit scale / min of sub-block j from the 12 packed bytes:
 * ggml-quants.c:818-825 (get_scale_min_k4). */
static inline void unpack_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* ggml-quants.c:1395-1465 (quantize_row_q4_K_ref) */
void bho_quantize_row_q4k(const float *x, void *vy, int64_t k) {
    uint8_t *y = (uint8_t *)vy;
    const int64_t nb = k / BHO_QK;
    uint8_t L[BHO_QK];
    float wts[32], sub_scale[8], sub_min[8];

    for (int64_t i = 0; i < nb; ++i, x += BHO_QK, y += BHO_Q4K_BYTES) {
        uint8_t *scales = y + 4;
        uint8_t *qs = y + 16;
        float max_scale = 0, max_min = 0;
        for (int j = 0; j < 8; ++j) {
            const float *xs = x + 32 * j;
            float ss = 0;
            for (int l = 0; l < 32; ++l) ss += xs[l] * xs[l];
            const float av = sqrtf(ss / 32);
            for (int l = 0; l < 32; ++l) wts[l] = av + fabsf(xs[l]);
            sub_scale[j] = fit_subblock(xs, wts, L + 32 * j, &sub_min[j]);
            if (sub_scale[j] > max_scale) max_scale = sub_scale[j];
            if (sub_min[j] > max_min) max_min = sub_min[j];
        }
        const float inv_scale = max_scale > 0 ? 63.f / max_scale : 0.f;
        const float inv_min = max_min > 0 ? 63.f / max_min : 0.f;
        for (int j = 0; j < 8; ++j) {
            uint8_t ls = (uint8_t)round_biased(inv_scale * sub_scale[j]);
            uint8_t lm = (uint8_t)round_biased(inv_min * sub_min[j]);
            if (ls > 63) ls = 63;
            if (lm > 63) lm = 63;
            if (j < 4) {
                scales[j] = ls;
                scales[j + 4] = lm;
            } else {
                scales[j + 4] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
                scales[j - 4] |= (uint8_t)((ls >> 4) << 6);
                scales[j] |= (uint8_t)((lm >> 4) << 6);
            }
        }
        const uint16_t hd = bho_fp32_to_fp16(max_scale / 63.f);
        const uint16_t hm = bho_fp32_to_fp16(max_min / 63.f);
        memcpy(y, &hd, 2);
        memcpy(y + 2, &hm, 2);

        const float fd = bho_fp16_to_fp32(hd), fm = bho_fp16_to_fp32(hm);
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            unpack_scale_min(j, scales, &sc, &mn);
            const float d = fd * sc;
            if (!d) continue; /* keeps the codes of fit_subblock */
            const float dm = fm * mn;
            for (int t = 0; t < 32; ++t) {
                int l = round_biased((x[32 * j + t] + dm) / d);
                L[32 * j + t] = (uint8_t)(l < 0 ? 0 : (l > 15 ? 15 : l));
            }
        }
        for (int g = 0; g < 4; ++g)
            for (int t = 0; t < 32; ++t)
                qs[32 * g + t] = (uint8_t)(L[64 * g + t] | (L[64 * g + 32 + t] << 4));
    }
}

typedef struct {
    const float *x;
    uint8_t *y;
    int64_t r0, r1, n_per_row;
} q4k_job;

static void *q4k_worker(void *arg) {
    const q4k_job *j = (const q4k_job *)arg;
    const int64_t rowb = j->n_per_row / BHO_QK * BHO_Q4K_BYTES;
    for (int64_t r = j->r0; r < j->r1; ++r)
        bho_quantize_row_q4k(j->x + r * j->n_per_row, j->y + r * rowb, j->n_per_row);
    return NULL;
}

void bho_quantize_q4k(const float *x, void *y, int64_t nrow, int64_t n_per_row, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > nrow) nthreads = (int)(nrow > 0 ? nrow : 1);
    pthread_t th[256];
    q4k_job jobs[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t].x = x;
        jobs[t].y = (uint8_t *)y;
        jobs[t].n_per_row = n_per_row;
        jobs[t].r0 = nrow * t / nthreads;
        jobs[t].r1 = nrow * (t + 1) / nthreads;
    }
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, q4k_worker, &jobs[t]);
    q4k_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

/* ggml-quants.c:1467-1489 (dequantize_row_q4_K) */
void bho_dequantize_row_q4k(const void *vx, float *y, int64_t k) {
    const uint8_t *x = (const uint8_t *)vx;
    const int64_t nb = k / BHO_QK;
    for (int64_t i = 0; i < nb; ++i, x += BHO_Q4K_BYTES) {
        const float d = bho_fp16_to_fp32(rd16(x));
        const float mnv = bho_fp16_to_fp32(rd16(x + 2));
        const uint8_t *q = x + 16;
        for (int g = 0; g < 4; ++g, q += 32) {
            int sc, mn;
            unpack_scale_min(2 * g, x + 4, &sc, &mn);
            const float d1 = d * sc, m1 = mnv * mn;
            unpack_scale_min(2 * g + 1, x + 4, &sc, &mn);
            const float d2 = d * sc, m2 = mnv * mn;
            for (int t = 0; t < 32; ++t) *y++ = d1 * (q[t] & 0xF) - m1;
            for (int t = 0; t < 32; ++t) *y++ = d2 * (q[t] >> 4) - m2;
        }
    }
}

/* ------------------------------------------------------------------ */
/* Q8_K quantizer: ggml-quants.c:2692-2729 (quantize_row_q8_K_ref)     */
/* ------------------------------------------------------------------ */
void bho_quantize_row_q8k(const float *x, void *vy, int64_t k) {
    uint8_t *y = (uint8_t *)vy;
    const int64_t nb = k / BHO_QK;
    for (int64_t i = 0; i < nb; ++i, x += BHO_QK, y += BHO_Q8K_BYTES) {
        int8_t *qs = (int8_t *)(y + 4);
        float amax = 0, vmax = 0;
        for (int t = 0; t < BHO_QK; ++t) {
            const float ax = fabsf(x[t]);
            if (ax > amax) { amax = ax; vmax = x[t]; }
        }
        if (!amax) {
            const float z = 0;
            memcpy(y, &z, 4);
            memset(y + 4, 0, BHO_Q8K_BYTES - 4); /* reference leaves bsums untouched */
            continue;
        }
        const float iscale = -127.f / vmax;
        for (int t = 0; t < BHO_QK; ++t) {
            const int v = round_biased(iscale * x[t]);
            qs[t] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int t = 0; t < 16; ++t) s += qs[16 * g + t];
            const int16_t s16 = (int16_t)s;
            memcpy(y + 260 + 2 * g, &s16, 2);
        }
        const float d = 1 / iscale;
        memcpy(y, &d, 4);
    }
}

/* ------------------------------------------------------------------ */
/* dot products                                                        */
/* ------------------------------------------------------------------ */

/* The 8 six-bit scales and 8 six-bit mins of one Q4_K block, as the
 * vec_dot kernels decode them (ggml-cpu/quants.c:685-690). */
static inline void decode_scales(const uint8_t *s12, int sc[8], int mn[8]) {
    for (int j = 0; j < 8; ++j) unpack_scale_min(j, s12, &sc[j], &mn[j]);
}

/* ggml-cpu/quants.c:645-718 (ggml_vec_dot_q4_K_q8_K_generic).
 * Lane l of the eight int32 accumulators collects the positions p of the
 * super-block with p % 8 == l; the fp32 fold is
 *   sums[l] += (fp16(d) * y.d) * aux32[l];  sumf -= (fp16(dmin) * y.d) * sumi;
 * then sumf += sums[0..7] in order. */
float bho_vec_dot_generic(int n, const void *vw, const void *vx) {
    const uint8_t *w = (const uint8_t *)vw;
    const uint8_t *xq = (const uint8_t *)vx;
    const int nb = n / BHO_QK;
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0;
    for (int i = 0; i < nb; ++i, w += BHO_Q4K_BYTES, xq += BHO_Q8K_BYTES) {
        int sc[8], mn[8];
        decode_scales(w + 4, sc, mn);
        const uint8_t *qs = w + 16;
        const int8_t *q8 = (const int8_t *)(xq + 4);
        int32_t aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int p = 0; p < BHO_QK; ++p) {
            const int j = p >> 5;                      /* sub-block */
            const int g = p >> 6, hi = (p >> 5) & 1;   /* 32-byte group, nibble */
            const int code = hi ? (qs[32 * g + (p & 31)] >> 4) : (qs[32 * g + (p & 31)] & 0xF);
            aux[p & 7] += sc[j] * (code * q8[p]);
        }
        int sumi = 0;
        for (int g = 0; g < 16; ++g) sumi += rds16(xq + 260 + 2 * g) * mn[g / 2];
        const float yd = rdf32(xq);
        const float d = bho_fp16_to_fp32(rd16(w)) * yd;
        for (int l = 0; l < 8; ++l) sums[l] += d * (float)aux[l];
        const float dmin = bho_fp16_to_fp32(rd16(w + 2)) * yd;
        sumf -= dmin * (float)sumi;
    }
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

/* ggml-cpu/arch/x86/quants.c:1900-1983 (AVX2 branch of
 * ggml_vec_dot_q4_K_q8_K), restated lane by lane.
 * Lane m (0..7) of the int32 accumulator collects, in every 64-value group,
 * byte positions 4m..4m+3 of the low-nibble half and of the high-nibble half
 * (maddubs + madd pair adjacent bytes, then adjacent pairs). Per block:
 *   acc[m]   = fma(y.d*fp16(d), (float)sumi[m], acc[m])
 *   accm[k]  = fma(-y.d*fp16(dmin), (float)(mn[2k]*S[2k] + mn[2k+1]*S[2k+1]), accm[k])
 * with S[t] = bsums[2t] + bsums[2t+1]. Final horizontal sums follow
 * hsum_float_8 (arch/x86/quants.c:43-49) and the 4-lane movehl/movehdup sum. */
float bho_vec_dot_x86(int n, const void *vw, const void *vx) {
    const uint8_t *w = (const uint8_t *)vw;
    const uint8_t *xq = (const uint8_t *)vx;
    const int nb = n / BHO_QK;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float accm[4] = {0, 0, 0, 0};
    for (int i = 0; i < nb; ++i, w += BHO_Q4K_BYTES, xq += BHO_Q8K_BYTES) {
        const float yd = rdf32(xq);
        const float d = yd * bho_fp16_to_fp32(rd16(w));
        const float dmin = -yd * bho_fp16_to_fp32(rd16(w + 2));
        int sc[8], mn[8];
        decode_scales(w + 4, sc, mn);
        const uint8_t *qs = w + 16;
        const int8_t *q8 = (const int8_t *)(xq + 4);

        int32_t S[8];
        for (int t = 0; t < 8; ++t)
            S[t] = (int16_t)(rds16(xq + 260 + 4 * t) + rds16(xq + 262 + 4 * t));
        for (int k = 0; k < 4; ++k) {
            const int32_t prod = mn[2 * k] * S[2 * k] + mn[2 * k + 1] * S[2 * k + 1];
            accm[k] = fmaf(dmin, (float)prod, accm[k]);
        }
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int g = 0; g < 4; ++g) {
            for (int b = 0; b < 32; ++b) {
                const int m = b >> 2;
                sumi[m] += sc[2 * g] * ((qs[32 * g + b] & 0xF) * q8[64 * g + b]);
                sumi[m] += sc[2 * g + 1] * ((qs[32 * g + b] >> 4) * q8[64 * g + 32 + b]);
            }
        }
        for (int m = 0; m < 8; ++m) acc[m] = fmaf(d, (float)sumi[m], acc[m]);
    }
    const float h = ((acc[4] + acc[0]) + (acc[6] + acc[2])) + ((acc[5] + acc[1]) + (acc[7] + acc[3]));
    const float hm = (accm[0] + accm[2]) + (accm[1] + accm[3]);
    return h + hm;
}

/* ggml-cpu/arch/x86/quants.c:2288-2370 (AVX2 branch of
 * ggml_vec_dot_q6_K_q8_K), restated lane by lane. block_q6_K
 * (ggml-common.h:352-357): ql[128] low 4 bits, qh[64] high 2 bits,
 * scales[16] int8 (one per 16 values), fp16 d; 210 bytes per 256 values.
 * Per 128-value half j and 32-value vector x (is = 4j + x) the 6-bit codes are
 *   x=0: ql[64j + b] & 15 | (qh[32j + b] & 3) << 4
 *   x=1: ql[64j + 32 + b] & 15 | (qh[32j + b] >> 2 & 3) << 4
 *   x=2: ql[64j + b] >> 4 | (qh[32j + b] >> 4 & 3) << 4
 *   x=3: ql[64j + 32 + b] >> 4 | (qh[32j + b] >> 6) << 4
 * for bytes b = 0..31 against q8[128j + 32x + b]. Lane m of the int32
 * accumulator takes bytes 4m..4m+3 of every vector, scaled by scales[2 is]
 * (m < 4) or scales[2 is + 1] (m >= 4), minus 32 * (bsums[2m] scales[2m] +
 * bsums[2m+1] scales[2m+1]); then acc[m] = fma(y.d * fp16(d), (float)sumi[m],
 * acc[m]) and hsum_float_8 at the end. */
float bho_vec_dot_q6k_x86(int n, const void *vw, const void *vx) {
    const uint8_t *w = (const uint8_t *)vw;
    const uint8_t *xq = (const uint8_t *)vx;
    const int nb = n / BHO_QK;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < nb; ++i, w += BHO_Q6K_BYTES, xq += BHO_Q8K_BYTES) {
        const float d = rdf32(xq) * bho_fp16_to_fp32(rd16(w + 208));
        const uint8_t *ql = w, *qh = w + 128;
        const int8_t *sc = (const int8_t *)(w + 192);
        const int8_t *q8 = (const int8_t *)(xq + 4);
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 2; ++j)
            for (int x = 0; x < 4; ++x) {
                const int is = 4 * j + x;
                for (int b = 0; b < 32; ++b) {
                    const uint8_t lo = ql[64 * j + 32 * (x & 1) + b];
                    const int q = ((x & 2) ? (lo >> 4) : (lo & 15)) | (((qh[32 * j + b] >> (2 * x)) & 3) << 4);
                    const int m = b >> 2;
                    sumi[m] += sc[2 * is + (m >= 4)] * (q * q8[128 * j + 32 * x + b]);
                }
            }
        for (int m = 0; m < 8; ++m) {
            const int32_t sub = rds16(xq + 260 + 4 * m) * sc[2 * m] + rds16(xq + 262 + 4 * m) * sc[2 * m + 1];
            sumi[m] -= sub << 5;
            acc[m] = fmaf(d, (float)sumi[m], acc[m]);
        }
    }
    return ((acc[4] + acc[0]) + (acc[6] + acc[2])) + ((acc[5] + acc[1]) + (acc[7] + acc[3]));
}

typedef struct {
    const uint8_t *W;
    const uint8_t *X;
    float *Y;
    int64_t N, K, r0, r1;
    int B;
} q6_job;

static void *q6_worker(void *arg) {
    const q6_job *j = (const q6_job *)arg;
    const int64_t nb = j->K / BHO_QK;
    const int64_t wrow = nb * BHO_Q6K_BYTES, xcol = nb * BHO_Q8K_BYTES;
    for (int b = 0; b < j->B; ++b)
        for (int64_t r = j->r0; r < j->r1; ++r)
            j->Y[(int64_t)b * j->N + r] = bho_vec_dot_q6k_x86((int)j->K, j->W + r * wrow, j->X + b * xcol);
    return NULL;
}

/* Y[b][r] = W_q6k[r] . Xq[b] over nthreads threads (x86 fold). */
void bho_matvec_q6k(const void *W, int64_t N, int64_t K, const void *Xq, int B, float *Y, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > N) nthreads = (int)(N > 0 ? N : 1);
    pthread_t th[256];
    q6_job jobs[256];
    for (int t = 0; t < nthreads; ++t)
        jobs[t] = (q6_job){(const uint8_t *)W, (const uint8_t *)Xq, Y, N, K, N * t / nthreads, N * (t + 1) / nthreads, B};
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, q6_worker, &jobs[t]);
    q6_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ */
/* matvec, partials, argmax                                            */
/* ------------------------------------------------------------------ */

typedef struct {
    const uint8_t *W;
    const uint8_t *X;
    float *Y;
    int64_t N, K, r0, r1;
    int B, fold;
} mv_job;

static void *mv_worker(void *arg) {
    const mv_job *j = (const mv_job *)arg;
    const int64_t nb = j->K / BHO_QK;
    const int64_t wrow = nb * BHO_Q4K_BYTES, xcol = nb * BHO_Q8K_BYTES;
    for (int b = 0; b < j->B; ++b)
        for (int64_t r = j->r0; r < j->r1; ++r)
            j->Y[(int64_t)b * j->N + r] = j->fold == BHO_FOLD_GENERIC
                ? bho_vec_dot_generic((int)j->K, j->W + r * wrow, j->X + b * xcol)
                : bho_vec_dot_x86((int)j->K, j->W + r * wrow, j->X + b * xcol);
    return NULL;
}

void bho_matvec(const void *W, int64_t N, int64_t K, const void *Xq, int B,
                float *Y, int fold, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > N) nthreads = (int)(N > 0 ? N : 1);
    pthread_t th[256];
    mv_job jobs[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (mv_job){(const uint8_t *)W, (const uint8_t *)Xq, Y, N, K,
                           N * t / nthreads, N * (t + 1) / nthreads, B, fold};
    }
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, mv_worker, &jobs[t]);
    mv_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

void bho_partials(const void *vW, int64_t N, int64_t K, const void *vX, int B, int32_t *out) {
    const uint8_t *W = (const uint8_t *)vW;
    const uint8_t *X = (const uint8_t *)vX;
    const int64_t nb = K / BHO_QK;
    for (int b = 0; b < B; ++b)
        for (int64_t r = 0; r < N; ++r)
            for (int64_t i = 0; i < nb; ++i) {
                const uint8_t *w = W + (r * nb + i) * BHO_Q4K_BYTES;
                const uint8_t *x = X + ((int64_t)b * nb + i) * BHO_Q8K_BYTES;
                const int8_t *q8 = (const int8_t *)(x + 4);
                int32_t *o = out + (((int64_t)b * N + r) * nb + i) * 9;
                int sc[8], mn[8];
                decode_scales(w + 4, sc, mn);
                for (int j = 0; j < 8; ++j) {
                    const int g = j >> 1, hi = j & 1;
                    int32_t s = 0;
                    for (int t = 0; t < 32; ++t) {
                        const uint8_t byte = w[16 + 32 * g + t];
                        s += (hi ? byte >> 4 : byte & 0xF) * q8[32 * j + t];
                    }
                    o[j] = s;
                }
                int32_t m = 0;
                for (int j = 0; j < 8; ++j)
                    m += mn[j] * (rds16(x + 260 + 4 * j) + rds16(x + 262 + 4 * j));
                o[8] = m;
            }
}

int64_t bho_argmax(const float *v, int64_t n) {
    int64_t best = 0;
    float bv = v[0];
    for (int64_t i = 1; i < n; ++i)
        if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

/* ------------------------------------------------------------------ */
/* routed-expert FFN glue (desktop/engine/src/forward.cpp:1001-1118)   */
/* ------------------------------------------------------------------ */

/* exp as ggml's AVX2 kernel evaluates it, one lane of ggml_v_expf
 * (ggml-cpu/vec.h:1233-1271; the method of ARM's optimized-routines expf:
 * n = round(x / ln2) through the 1.5*2^23 shift, b = x - n*ln2 in two fused
 * steps, a degree-5 polynomial j ~ exp(b) - 1 in Estrin form, then
 * k = 2^n built in the exponent field and exp = k + k*j; |n| > 126 takes
 * the two-factor scaling s2*s1 so subnormal and overflowing results round
 * once, |n| > 192 saturates to s1*s1). Every step is one correctly
 * rounded binary32 operation, as the intrinsics are, so the GPU's
 * exp_ggml (csrc/bh_math.cuh) and the reference agree bit for bit.
 * The reference's scalar tails (n % 8 elements of soft_max, SiLU of
 * lengths not a multiple of 8) call libm expf instead. */
float bho_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float n = z - r;
    const float b = fmaf(-n, 0x1.7f7d1cp-20f, fmaf(-n, 0x1.62e4p-1f, x));
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + 0x3f800000u);
    const int c = fabsf(n) > 126.0f;
    const float u = b * b;
    const float j = fmaf(fmaf(fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u, fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                         u, 0x1.ffffecp-1f * b);
    if (!c) return fmaf(j, k, k);
    const uint32_t g = n <= 0.0f ? 0x82000000u : 0u;
    const float s1 = u2f(g + 0x7f000000u);
    const float s2 = u2f(e - g);
    if (fabsf(n) > 192.0f) return s1 * s1;
    return fmaf(s2, j, s2) * s1;
}

/* ggml_v_silu, one lane (ggml-cpu/vec.h:1273-1280, ggml_vec_silu_f32 at
 * vec.cpp:396): x / (1 + exp(0 - x)) */
float bho_silu(float x) { return x / (1.0f + bho_expf(0.0f - x)); }

void bho_expf_n(const float *x, int64_t n, float *y) { for (int64_t i = 0; i < n; ++i) y[i] = bho_expf(x[i]); }
void bho_silu_n(const float *x, int64_t n, float *y) { for (int64_t i = 0; i < n; ++i) y[i] = bho_silu(x[i]); }

/* ggml_compute_forward_rms_norm_f32 (ggml-cpu/ops.cpp): sum of the fp32
 * squares accumulated in double, mean = (float)(sum / n),
 * scale = 1 / sqrtf(mean + eps), y = x * scale; then the norm weight
 * (ggml_mul): y * gamma. gamma may be NULL (no weight). */
void bho_rmsnorm(const float *x, const float *gamma, int n, float eps, float *y) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) {
        const float v = x[i] * scale;
        y[i] = gamma ? v * gamma[i] : v;
    }
}

/* Router of one token:
 *  soft_max (ggml-cpu/ops.cpp:5365-5382 with vec.cpp:547-567, AVX2 branch):
 *    max; p_i = exp(l_i - max); sum in double of per-8 fp32 partial sums
 *    ((p4+p0)+(p6+p2)) + ((p5+p1)+(p7+p3)), tail added one by one;
 *    p_i *= (float)(1.0 / sum)
 *  top_k (ops.cpp:8157-8194): the k largest p in descending order, then
 *    slots 0 and 1 swapped. Equal p are taken lower index first (the
 *    reference's std::partial_sort leaves their order unspecified).
 *  get_rows + norm_topk_prob (forward.cpp:1032-1046): w_s = p[ids_s];
 *    w_s /= (float)(sum in double of w over the slots, in slot order). */
void bho_moe_route(const float *logits, int n_expert, int k, int norm, int32_t *ids, float *w) {
    float p[1024];
    float mx = -INFINITY;
    for (int i = 0; i < n_expert; ++i) mx = logits[i] > mx ? logits[i] : mx;
    for (int i = 0; i < n_expert; ++i) p[i] = bho_expf(logits[i] - mx);
    double sum = 0.0;
    int i = 0;
    for (; i + 7 < n_expert; i += 8) {
        const float *v = p + i;
        const float g = ((v[4] + v[0]) + (v[6] + v[2])) + ((v[5] + v[1]) + (v[7] + v[3]));
        sum += (double)g;
    }
    for (; i < n_expert; ++i) sum += (double)p[i];
    const float inv = (float)(1.0 / sum);
    for (i = 0; i < n_expert; ++i) p[i] *= inv;
    /* selection: rank by (p descending, index ascending) */
    for (int s = 0; s < k; ++s) {
        int best = -1;
        for (int e = 0; e < n_expert; ++e) {
            int taken = 0;
            for (int u = 0; u < s; ++u) taken |= ids[u] == e;
            if (taken) continue;
            if (best < 0 || p[e] > p[best]) best = e;
        }
        ids[s] = best;
    }
    if (k > 1) { const int32_t t = ids[0]; ids[0] = ids[1]; ids[1] = t; }
    for (int s = 0; s < k; ++s) w[s] = p[ids[s]];
    if (norm) {
        double ws = 0.0;
        for (int s = 0; s < k; ++s) ws += (double)w[s];
        const float wsf = (float)ws;
        for (int s = 0; s < k; ++s) w[s] = w[s] / wsf;
    }
}

/* Stock routed-expert FFN (forward.cpp:1090-1107) for T tokens:
 *   up_e = W_up[e] . q8k(cur_t),  gate_e = W_gate[e] . q8k(cur_t)   (mul_mat_id)
 *   par  = silu(gate_e) * up_e                                       (ggml_silu, ggml_mul)
 *   down = W_down[e] . q8k(par)                                      (mul_mat_id)
 *   out_t = (float) sum over slots s, in order, of (double)(down_s * w_s)
 *                                                  (ggml_mul, ggml_sum_rows)
 * Banks: gate/up [n_expert][n_ff rows][n_embd/256 blocks] and
 * down [n_expert][n_embd rows][n_ff/256 blocks] of block_q4_K.
 * gu_opt [T*k][2*n_ff] receives gate | up (before SiLU); dout_opt
 * [T*k][n_embd] the unweighted expert outputs. */
void bho_moe_ffn(const float *cur, int T, const int32_t *ids, const float *w, int k,
                 const void *gate, const void *up, const void *down, int n_embd, int n_ff,
                 float *out, float *gu_opt, float *dout_opt, int fold, int nthreads) {
    const int64_t nbe = n_embd / BHO_QK, nbf = n_ff / BHO_QK;
    const int64_t gsz = (int64_t)n_ff * nbe * BHO_Q4K_BYTES;     /* bytes of one gate/up expert */
    const int64_t dsz = (int64_t)n_embd * nbf * BHO_Q4K_BYTES;   /* bytes of one down expert */
    uint8_t *xq = (uint8_t *)malloc((size_t)nbe * BHO_Q8K_BYTES);
    uint8_t *pq = (uint8_t *)malloc((size_t)nbf * BHO_Q8K_BYTES);
    float *g = (float *)malloc(sizeof(float) * 2 * (size_t)n_ff);
    float *par = (float *)malloc(sizeof(float) * (size_t)n_ff);
    float *d = (float *)malloc(sizeof(float) * (size_t)n_embd);
    double *acc = (double *)malloc(sizeof(double) * (size_t)n_embd);
    for (int t = 0; t < T; ++t) {
        bho_quantize_row_q8k(cur + (int64_t)t * n_embd, xq, n_embd);
        for (int i = 0; i < n_embd; ++i) acc[i] = 0.0;
        for (int s = 0; s < k; ++s) {
            const int e = ids[t * k + s];
            bho_matvec((const uint8_t *)gate + e * gsz, n_ff, n_embd, xq, 1, g, fold, nthreads);
            bho_matvec((const uint8_t *)up + e * gsz, n_ff, n_embd, xq, 1, g + n_ff, fold, nthreads);
            if (gu_opt) memcpy(gu_opt + ((int64_t)t * k + s) * 2 * n_ff, g, sizeof(float) * 2 * (size_t)n_ff);
            for (int i = 0; i < n_ff; ++i) par[i] = bho_silu(g[i]) * g[n_ff + i];
            bho_quantize_row_q8k(par, pq, n_ff);
            bho_matvec((const uint8_t *)down + e * dsz, n_embd, n_ff, pq, 1, d, fold, nthreads);
            if (dout_opt) memcpy(dout_opt + ((int64_t)t * k + s) * n_embd, d, sizeof(float) * (size_t)n_embd);
            const float ws = w[t * k + s];
            for (int i = 0; i < n_embd; ++i) acc[i] += (double)(d[i] * ws);
        }
        for (int i = 0; i < n_embd; ++i) out[(int64_t)t * n_embd + i] = (float)acc[i];
    }
    free(xq); free(pq); free(g); free(par); free(d); free(acc);
}
