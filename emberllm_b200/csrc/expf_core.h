/* expf_core.h — the exp recipe shared bit-for-bit by host (C11) and device (CUDA).
 *
 * The reference computes expf with the host C library (softmax, ref
 * src/model.c:61; SiLU, ref src/model.c:405), and its logits depend on every bit
 * of it. This file does not reproduce any library's expf. It evaluates exp(x) in
 * double precision with a textbook table-driven recipe:
 *
 *   k = nearest integer to x*64/ln2 (by the 1.5*2^52 shifter trick),
 *   r = (x - k*hi) - k*lo, hi + lo = ln2/64   (Cody & Waite range reduction),
 *   P(r) = sum_{j<=5} r^j/j! by Horner        (|r| <= ln2/128),
 *   exp(x) = P(r) * 2^((k mod 64)/64) * 2^floor(k/64),
 *
 * with 2^(j/64) from a 64-entry table the host fills, and rounds the double to
 * float. Its error is ~1e-8 float ulp, so it equals the
 * correctly rounded expf except very near a rounding midpoint. Where the C
 * library's result differs from it (it is within ~0.5 ulp but not always
 * correctly rounded), the input is listed in an exception table that the host
 * builds by scanning every float input once on the machine that runs the model
 * (csrc/host/tables.c). All constants come from EmberExpfParams, filled by the
 * host, so both sides compute with identical bits; the host is compiled with
 * -ffp-contract=off and the device spells every operation with _rn intrinsics,
 * so neither side fuses multiply-adds.
 */
#ifndef EMBER_B200_EXPF_CORE_H
#define EMBER_B200_EXPF_CORE_H

#include "ember_cuda.h"

#if defined(__CUDACC__)
#  define EXC_FN static __host__ __device__ __forceinline__
#else
#  define EXC_FN static inline
#endif

#if defined(__CUDA_ARCH__)
#  define EXC_ADD(a, b) __dadd_rn((a), (b))
#  define EXC_MUL(a, b) __dmul_rn((a), (b))
#  define EXC_D2F(y) __double2float_rn(y)
#else
#  define EXC_ADD(a, b) ((a) + (b))
#  define EXC_MUL(a, b) ((a) * (b))
#  define EXC_D2F(y) ((float)(y))
#endif

EXC_FN uint32_t exc_fbits(float f) { union { float f; uint32_t u; } c; c.f = f; return c.u; }
EXC_FN float exc_bitsf(uint32_t u) { union { float f; uint32_t u; } c; c.u = u; return c.f; }

/* exp(x) in double by the recipe above with the 2^(j/64) table at `tab` (the
 * device keeps a copy in shared memory); x finite and within [p->lo, p->hi] */
EXC_FN double exc_exp_double_t(const EmberExpfParams *p, const double *tab, float xf) {
    double x = (double)xf;
    double t = EXC_ADD(EXC_MUL(x, p->inv_step), p->shifter);
    double kd = EXC_ADD(t, -p->shifter);
    int k = (int)kd;
    double r = EXC_ADD(EXC_ADD(x, -EXC_MUL(kd, p->step_hi)), -EXC_MUL(kd, p->step_lo));
    double q = p->coef[5];
    for (int j = 4; j >= 0; j--) q = EXC_ADD(EXC_MUL(q, r), p->coef[j]);
    int j = k & 63, m = (k - j) / 64;
    union { unsigned long long u; double d; } s;
    s.u = (unsigned long long)((long long)m + 1023) << 52;
    return EXC_MUL(EXC_MUL(q, tab[j]), s.d);
}

EXC_FN double exc_exp_double(const EmberExpfParams *p, float xf) { return exc_exp_double_t(p, p->tab, xf); }

EXC_FN unsigned long long exc_dbits(double d) { union { double d; unsigned long long u; } c; c.d = d; return c.u; }

/* distance of a double y (whose float rounding r is normal, not FLT_MIN or
 * FLT_MAX) from the nearest float rounding midpoint, in units of 2^-29 float ulp:
 * the low 29 bits of y's mantissa are its position inside one float ulp */
EXC_FN unsigned exc_mid_distance(double y) {
    long long low = (long long)(exc_dbits(y) & ((1ull << 29) - 1)) - (1ll << 28);
    return (unsigned)(low < 0 ? -low : low);
}

/* Round y (> 0) to float. *flag is set when the result may need the exception
 * table: y within the window of a rounding midpoint, or a result that is not a
 * normal float strictly between FLT_MIN and FLT_MAX. */
EXC_FN float exc_round(const EmberExpfParams *p, double y, int *flag) {
    float r = EXC_D2F(y);
    uint32_t rb = exc_fbits(r);
    if (rb >= 0x7F7FFFFFu || rb <= 0x00800000u) { *flag = 1; return r; }
    *flag = exc_mid_distance(y) < p->window;
    return r;
}

EXC_FN uint32_t exc_hash(uint32_t xb, uint32_t n_slots) {
    return (xb * 0x9E3779B1u) & (n_slots - 1u);
}

/* The full function: the C library's expf(x), given the host-built tables. */
EXC_FN float exc_expf_t(const EmberExpfParams *p, const double *tab, const uint32_t *slots, float x) {
    if (x != x) return x + x;
    if (x < p->lo) return 0.0f;
    if (x > p->hi) return exc_bitsf(0x7F800000u);
    int flag = 0;
    float r = exc_round(p, exc_exp_double_t(p, tab, x), &flag);
    if (flag) {
        uint32_t xb = exc_fbits(x);
        uint32_t i = exc_hash(xb, p->n_slots);
        /* the table is at most half full, so an empty slot ends the probe early */
        for (uint32_t probe = 0; probe < p->n_slots; probe++) {
            uint32_t key = slots[2u * i];
            if (key == xb) return exc_bitsf(slots[2u * i + 1u]);
            if (key == EMBER_EXPF_EMPTY) break;
            i = (i + 1u) & (p->n_slots - 1u);
        }
    }
    return r;
}

EXC_FN float exc_expf(const EmberExpfParams *p, const uint32_t *slots, float x) {
    return exc_expf_t(p, p->tab, slots, x);
}

#endif /* EMBER_B200_EXPF_CORE_H */
