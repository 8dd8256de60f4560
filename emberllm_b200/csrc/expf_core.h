/* expf_core.h — the exp recipe shared bit-for-bit by host (C11) and device (CUDA).
 *
 * The reference computes expf with the host C library (softmax, ref
 * src/model.c:61; SiLU, ref src/model.c:405), and its logits depend on every bit
 * of it. This file does not reproduce any library's expf. It evaluates exp(x) in
 * double precision with a textbook recipe:
 *
 *   k = nearest integer to x/ln2 (by the 1.5*2^52 shifter trick),
 *   r = (x - k*ln2_hi) - k*ln2_lo            (Cody & Waite range reduction),
 *   exp(r) by Horner on the degree-12 Taylor polynomial sum r^j/j!,
 *   exp(x) = exp(r) * 2^k,
 *
 * and rounds the double to float. Its error is ~1e-8 float ulp, so it equals the
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

/* exp(x) in double by the recipe above; x finite and within [p->lo, p->hi] */
EXC_FN double exc_exp_double(const EmberExpfParams *p, float xf) {
    double x = (double)xf;
    double t = EXC_ADD(EXC_MUL(x, p->inv_ln2), p->shifter);
    double k = EXC_ADD(t, -p->shifter);
    double r = EXC_ADD(EXC_ADD(x, -EXC_MUL(k, p->ln2_hi)), -EXC_MUL(k, p->ln2_lo));
    double q = p->coef[12];
    for (int j = 11; j >= 0; j--) q = EXC_ADD(EXC_MUL(q, r), p->coef[j]);
    union { unsigned long long u; double d; } s;
    s.u = (unsigned long long)((long long)k + 1023) << 52;
    return EXC_MUL(q, s.d);
}

/* Round y (> 0) to float. *flag is set when the result may need the exception
 * table: y within p->delta ulps of a rounding midpoint, or a result that is not
 * a normal float below FLT_MAX. */
EXC_FN float exc_round(const EmberExpfParams *p, double y, int *flag) {
    float r = EXC_D2F(y);
    uint32_t rb = exc_fbits(r);
    if (rb >= 0x7F7FFFFFu || rb < 0x00800000u) { *flag = 1; return r; }
    double rd = (double)r;
    uint32_t nb = (y >= rd) ? rb + 1u : rb - 1u;
    double nd = (double)exc_bitsf(nb);
    double mid = EXC_MUL(EXC_ADD(rd, nd), 0.5);
    double ulp = nd > rd ? EXC_ADD(nd, -rd) : EXC_ADD(rd, -nd);
    double dist = EXC_ADD(y, -mid);
    if (dist < 0) dist = -dist;
    *flag = dist < EXC_MUL(p->delta, ulp);
    return r;
}

/* distance of y from the nearest midpoint in ulps (host table builder only) */
EXC_FN double exc_midpoint_ulps(double y, float r) {
    uint32_t rb = exc_fbits(r);
    double rd = (double)r;
    uint32_t nb = (y >= rd) ? rb + 1u : rb - 1u;
    double nd = (double)exc_bitsf(nb);
    double mid = EXC_MUL(EXC_ADD(rd, nd), 0.5);
    double ulp = nd > rd ? EXC_ADD(nd, -rd) : EXC_ADD(rd, -nd);
    double dist = EXC_ADD(y, -mid);
    if (dist < 0) dist = -dist;
    return dist / ulp;
}

EXC_FN uint32_t exc_hash(uint32_t xb, uint32_t n_slots) {
    return (xb * 0x9E3779B1u) & (n_slots - 1u);
}

/* The full function: the C library's expf(x), given the host-built table. */
EXC_FN float exc_expf(const EmberExpfParams *p, const uint32_t *slots, float x) {
    if (x != x) return x + x;
    if (x < p->lo) return 0.0f;
    if (x > p->hi) return exc_bitsf(0x7F800000u);
    int flag = 0;
    float r = exc_round(p, exc_exp_double(p, x), &flag);
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

#endif /* EMBER_B200_EXPF_CORE_H */
