/* quant.c — host-side fp16 conversion, block quantizers and the offline
 * requantizer (replaces ref src/kernels.c:25-115 and src/quant.c:59-125).
 *
 * These run on the CPU because they produce the .ember file format offline;
 * the token loop's activation quantization is done on the GPU (quant_quad and
 * quant_lane in csrc/cuda/common.cuh). Every rounding step here follows the reference bit for
 * bit, because the file bytes they produce are what both the reference and this
 * library then read: the tests compare ember_quantize_file's output byte for byte
 * against emberllm's `ember quantize`. Build with -ffp-contract=off.
 */
#include "ember_ops.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* binary16 -> binary32: exact (ref src/kernels.c:25-46). */
float ember_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0x1Fu) return bits_f32(sign | 0x7F800000u | (m << 13));    /* inf / nan */
    if (e != 0) return bits_f32(sign | ((e + 112u) << 23) | (m << 13)); /* normal */
    if (m == 0) return bits_f32(sign);                                   /* +-0 */
    /* subnormal half: value = m * 2^-24; renormalise into a float */
    int shift = 0;
    while ((m & 0x400u) == 0) { m <<= 1; shift++; }
    return bits_f32(sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3FFu) << 13));
}

/* binary32 -> binary16, round to nearest, ties to even (ref src/kernels.c:48-68).
 * Like the reference, a NaN input maps to infinity. */
uint16_t ember_f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    uint32_t e = ax >> 23;               /* biased float exponent */
    uint32_t m = ax & 0x7FFFFFu;
    if (e >= 143u) return sign | 0x7C00u; /* |f| >= 2^16, inf, nan: overflow */
    if (e >= 113u) {                      /* normal half range before rounding */
        uint32_t h = ((e - 112u) << 10) | (m >> 13);
        uint32_t rest = m & 0x1FFFu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++; /* may carry to inf */
        return (uint16_t)(sign | h);
    }
    if (e < 102u) return sign;            /* below 2^-25: rounds to zero */
    /* subnormal half: value in units of 2^-24 is (m|hidden) >> (126 - e) */
    uint32_t full = m | 0x800000u;
    uint32_t sh = 126u - e;               /* 14..24 */
    uint32_t h = full >> sh;
    uint32_t rest = full & ((1u << sh) - 1u);
    uint32_t halfway = 1u << (sh - 1u);
    if (rest > halfway || (rest == halfway && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* Q8_0 (ref src/kernels.c:73-92): per 32-block d = max|x| / 127, q = round-half-
 * away(x * (1/d)) clamped to +-127, d stored as fp16. */
void ember_quantize_q8_0(const float *x, BlockQ8_0 *out, int n) {
    for (int b = 0; b < n / EMBER_Q_BLOCK; b++) {
        const float *v = x + (size_t)b * EMBER_Q_BLOCK;
        float amax = 0.0f;
        for (int i = 0; i < EMBER_Q_BLOCK; i++) {
            float a = fabsf(v[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float inv = d > 0.0f ? 1.0f / d : 0.0f;
        out[b].d = ember_f32_to_f16(d);
        for (int i = 0; i < EMBER_Q_BLOCK; i++) {
            long q = lroundf(v[i] * inv);
            out[b].qs[i] = (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
        }
    }
}

/* Q4_0 (ref src/kernels.c:95-115): d = (the value of largest magnitude, first one
 * on ties) / -8; nibble = trunc(x/d + 8.5) clamped to [0,15]; byte i packs
 * element i (low nibble) with element i+16 (high nibble). */
void ember_quantize_q4_0(const float *x, BlockQ4_0 *out, int n) {
    for (int b = 0; b < n / EMBER_Q_BLOCK; b++) {
        const float *v = x + (size_t)b * EMBER_Q_BLOCK;
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < EMBER_Q_BLOCK; i++) {
            float a = fabsf(v[i]);
            if (a > amax) { amax = a; vmax = v[i]; }
        }
        float d = vmax / -8.0f;
        float inv = d != 0.0f ? 1.0f / d : 0.0f;
        out[b].d = ember_f32_to_f16(d);
        for (int i = 0; i < EMBER_Q_BLOCK / 2; i++) {
            int lo = (int)(v[i] * inv + 8.5f);
            int hi = (int)(v[i + EMBER_Q_BLOCK / 2] * inv + 8.5f);
            lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
            hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
            out[b].qs[i] = (uint8_t)(lo | (hi << 4));
        }
    }
}

/* ---- offline requantizer ------------------------------------------------ */

static uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

typedef struct {
    EmberTensor meta;
    void *bytes;
    uint64_t size;
} Staged;

static int stage_tensor(const EmberTensor *t, const void *src, int target, Staged *o) {
    o->meta = *t;
    int want = target;
    if (target == EMBER_DT_Q4_0 &&
        (strcmp(t->name, "tok_embeddings") == 0 || strcmp(t->name, "lm_head") == 0))
        want = EMBER_DT_Q8_0;                      /* ref src/quant.c:71-75 */
    int rows = t->shape[0], cols = t->shape[1];
    int quantize = t->dtype == EMBER_DT_F32 && t->ndim >= 2 && cols % EMBER_Q_BLOCK == 0 &&
                   want != EMBER_DT_F32;
    if (t->dtype != EMBER_DT_F32 || !quantize) {   /* copy through unchanged */
        o->size = t->nbytes;
        o->bytes = malloc(o->size ? o->size : 1);
        if (!o->bytes) return 1;
        memcpy(o->bytes, src, o->size);
        return 0;
    }
    const float *f = (const float *)src;
    int nb = cols / EMBER_Q_BLOCK;
    if (want == EMBER_DT_Q4_0) {
        o->meta.dtype = EMBER_DT_Q4_0;
        o->size = (uint64_t)rows * nb * sizeof(BlockQ4_0);
        BlockQ4_0 *q = malloc(o->size);
        if (!q) return 1;
        for (int r = 0; r < rows; r++)
            ember_quantize_q4_0(f + (size_t)r * cols, q + (size_t)r * nb, cols);
        o->bytes = q;
    } else {
        o->meta.dtype = EMBER_DT_Q8_0;
        o->size = (uint64_t)rows * nb * sizeof(BlockQ8_0);
        BlockQ8_0 *q = malloc(o->size);
        if (!q) return 1;
        for (int r = 0; r < rows; r++)
            ember_quantize_q8_0(f + (size_t)r * cols, q + (size_t)r * nb, cols);
        o->bytes = q;
    }
    return 0;
}

static int write_zeros(FILE *f, uint64_t upto) {
    static const char zeros[64] = {0};
    long at = ftell(f);
    if (at < 0) return 1;
    uint64_t cur = (uint64_t)at;
    while (cur < upto) {
        uint64_t k = upto - cur > sizeof(zeros) ? sizeof(zeros) : upto - cur;
        if (fwrite(zeros, 1, k, f) != k) return 1;
        cur += k;
    }
    return 0;
}

/* Same layout rules as ref src/quant.c:86-117: header, tokenizer blob at 256,
 * table 8-aligned after it, data region and every tensor 64-aligned. */
int ember_quantize_file(const char *in_path, const char *out_path, int target) {
    EmberModel *m = ember_model_load(in_path);
    if (!m) return 1;
    const EmberHeader *h = ember_model_header(m);
    const EmberTensor *table =
        (const EmberTensor *)((const uint8_t *)h + h->tensor_table_offset);
    int n = h->n_tensors;
    Staged *st = calloc(n > 0 ? (size_t)n : 1, sizeof(Staged));
    int rc = st ? 0 : 1;
    for (int i = 0; i < n && rc == 0; i++) {
        const void *src = ember_model_data(m, &table[i]);
        rc = src ? stage_tensor(&table[i], src, target, &st[i]) : 1;
    }
    FILE *f = NULL;
    uint64_t end = 0;
    if (rc == 0) {
        EmberHeader nh = *h;
        uint64_t tok_off = sizeof(EmberHeader);
        uint64_t table_off = round_up(tok_off + h->tokenizer_size, 8);
        uint64_t table_size = (uint64_t)n * sizeof(EmberTensor);
        uint64_t data_off = round_up(table_off + table_size, 64);
        end = data_off;
        for (int i = 0; i < n; i++) {
            end = round_up(end, 64);
            st[i].meta.offset = end;
            st[i].meta.nbytes = st[i].size;
            end += st[i].size;
        }
        nh.header_bytes = data_off;
        nh.tokenizer_offset = tok_off;
        nh.tensor_table_offset = table_off;
        nh.tensor_table_size = table_size;
        f = fopen(out_path, "wb");
        if (!f) rc = 1;
        if (rc == 0 && fwrite(&nh, sizeof(nh), 1, f) != 1) rc = 1;
        if (rc == 0 && h->tokenizer_size &&
            fwrite((const uint8_t *)h + h->tokenizer_offset, 1, h->tokenizer_size, f) !=
                h->tokenizer_size)
            rc = 1;
        if (rc == 0) rc = write_zeros(f, table_off);
        for (int i = 0; i < n && rc == 0; i++)
            if (fwrite(&st[i].meta, sizeof(EmberTensor), 1, f) != 1) rc = 1;
        if (rc == 0) rc = write_zeros(f, data_off);
        for (int i = 0; i < n && rc == 0; i++) {
            rc = write_zeros(f, st[i].meta.offset);
            if (rc == 0 && st[i].size && fwrite(st[i].bytes, 1, st[i].size, f) != st[i].size) rc = 1;
        }
        if (f && fclose(f) != 0) rc = 1;
    }
    if (rc == 0) fprintf(stderr, "quantized %s -> %s (%.1f MB)\n", in_path, out_path, end / 1e6);
    if (st) for (int i = 0; i < n; i++) free(st[i].bytes);
    free(st);
    ember_model_free(m);
    return rc;
}
