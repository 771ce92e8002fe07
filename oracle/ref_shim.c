/*
 * ref_shim.c — the handful of ggml core symbols that the reference's quant
 * sources reference, so that ggml-quants.c, ggml-cpu/quants.c and
 * ggml-cpu/arch/x86/quants.c link into oracle/_ref without building the
 * rest of ggml. TEST INFRASTRUCTURE ONLY.
 *
 * Only the Q4_K / Q8_K paths are exercised; the type helpers answer for
 * those two types and abort on anything else.
 */
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "q4k_oracle.h"

/* ggml type ids (vendor/ggml/include/ggml.h enum ggml_type) */
#define REF_TYPE_Q4_K 12
#define REF_TYPE_Q8_K 15

float ggml_table_f32_f16[1 << 16];
float ggml_table_f32_e8m0_half[1 << 8];

__attribute__((constructor)) static void ref_shim_init(void) {
    for (uint32_t h = 0; h < (1u << 16); ++h) ggml_table_f32_f16[h] = bho_fp16_to_fp32((uint16_t)h);
    for (uint32_t e = 0; e < 256; ++e) {
        /* e8m0 value 2^(e-127), halved; not on the Q4_K path */
        uint32_t bits = e < 2 ? (0x00200000u << e) : ((e - 1) << 23);
        memcpy(&ggml_table_f32_e8m0_half[e], &bits, 4);
    }
}

void ggml_abort(const char *file, int line, const char *fmt, ...) {
    va_list ap;
    fprintf(stderr, "ggml_abort %s:%d: ", file, line);
    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
    fputc('\n', stderr);
    abort();
}

size_t ggml_type_size(int type) {
    if (type == REF_TYPE_Q4_K) return 144;
    if (type == REF_TYPE_Q8_K) return 292;
    ggml_abort(__FILE__, __LINE__, "ref shim: type %d not supported", type);
    return 0;
}

const char *ggml_type_name(int type) {
    if (type == REF_TYPE_Q4_K) return "q4_K";
    if (type == REF_TYPE_Q8_K) return "q8_K";
    return "unsupported";
}

size_t ggml_row_size(int type, int64_t ne) { return ggml_type_size(type) * (size_t)(ne / 256); }
