/* exact_sum_core.h — the pieces of a PARALLEL evaluation of a SEQUENTIAL fp32 sum
 * of non-negative terms, bit-identical to the reference's loop
 *
 *     float s = 0; for (i = 0; i < n; i++) s += p[i];      (round to nearest even)
 *
 * (its RMSNorm sum of squares, ref src/model.c:52, and softmax denominator,
 * ref src/model.c:61). Shared by the device kernels and the host tests.
 *
 * Why it works. While the running sum s stays in one binade [2^e, 2^(e+1)) its
 * spacing u = 2^(e-23) is fixed, so one step is s + p rounded to the grid of u:
 * s + u*k with k = round(p/u); only an exact tie (p/u = n + 1/2) depends on s,
 * through the parity of s/u. A step is therefore the pair (A, B) = (k if s/u is
 * even, k if s/u is odd), and pairs compose associatively:
 *
 *     (A1,B1) then (A2,B2) = (A1 + (A1 odd ? B2 : A2),  B1 + (B1 odd ? A2 : B2)).
 *
 * The terms are non-negative, so the float running sum s_i stays within
 * (i-1)*2^-24 (relative) of the exact prefix sum, which a double-precision
 * parallel prefix gives to ~1e-13. Where that interval lies inside one binade
 * for both s_i and s_{i+1}, step i is such a pair ("run" step); the few other
 * steps (binade crossings, tiny or zero sums) are done as ordinary float
 * additions in order. Runs between those steps are composed in parallel.
 */
#ifndef EMBER_B200_EXACT_SUM_CORE_H
#define EMBER_B200_EXACT_SUM_CORE_H

#include <stdint.h>

#if defined(__CUDACC__)
#  define XS_FN static __host__ __device__ __forceinline__
#else
#  define XS_FN static inline
#endif

#if defined(__CUDA_ARCH__)
#  define XS_DADD(a, b) __dadd_rn((a), (b))
#  define XS_DMUL(a, b) __dmul_rn((a), (b))
#  define XS_FADD(a, b) __fadd_rn((a), (b))
#else
#  define XS_DADD(a, b) ((a) + (b))
#  define XS_DMUL(a, b) ((a) * (b))
#  define XS_FADD(a, b) ((a) + (b))
#endif

#define XS_NO_BINADE (-1000)   /* binade unknown (or not a normal float range) */

typedef struct { int e, a, b; } XsRun;   /* composed run in binade e (e = XS_NO_BINADE: empty) */

XS_FN uint64_t xs_dbits(double d) { union { double d; uint64_t u; } c; c.d = d; return c.u; }
XS_FN double xs_bitsd(uint64_t u) { union { double d; uint64_t u; } c; c.u = u; return c.d; }
XS_FN uint32_t xs_fbits(float f) { union { float f; uint32_t u; } c; c.f = f; return c.u; }
XS_FN float xs_bitsf(uint32_t u) { union { float f; uint32_t u; } c; c.u = u; return c.f; }

/* floor(log2(d)) for a positive normal double */
XS_FN int xs_dexp(double d) { return (int)((xs_dbits(d) >> 52) & 0x7FF) - 1023; }

/* The binade e of the float running sum after `i` additions, known to lie
 * within a relative (i+2)*6e-8 of the exact prefix D (which itself is within
 * ~1e-13); XS_NO_BINADE unless the whole interval is inside one normal binade
 * comfortably away from the extremes. */
XS_FN int xs_certain_binade(double D, int i) {
    if (!(D >= 0x1p-100) || !(D < 0x1p126)) return XS_NO_BINADE;
    double g = (double)(i + 2) * 6.0e-8;
    double lo = XS_DMUL(D, XS_DADD(1.0, -g)), hi = XS_DMUL(D, XS_DADD(1.0, g));
    int elo = xs_dexp(lo), ehi = xs_dexp(hi);
    return elo == ehi ? elo : XS_NO_BINADE;
}

/* the pair (A, B) of one step adding p (>= 0) to a running sum in binade e */
XS_FN void xs_step_pair(float p, int e, int *A, int *B) {
    double u = xs_bitsd((uint64_t)(e - 23 + 1023) << 52);   /* 2^(e-23), exact */
    double m = (double)p / u;                                  /* exact: power-of-two scaling */
    double n = (double)(int64_t)m;                              /* m >= 0: truncation = floor */
    double f = XS_DADD(m, -n);
    int ni = (int)n;
    if (f < 0.5) { *A = ni; *B = ni; }
    else if (f > 0.5) { *A = ni + 1; *B = ni + 1; }
    else {                                  /* exact tie: the result mantissa must be even */
        *A = (ni & 1) ? ni + 1 : ni;        /* s/u even: k even */
        *B = (ni & 1) ? ni : ni + 1;        /* s/u odd:  k odd  */
    }
}

XS_FN XsRun xs_empty(void) { XsRun r; r.e = XS_NO_BINADE; r.a = 0; r.b = 0; return r; }

/* r1 then r2 (both in the same binade, or either empty) */
XS_FN XsRun xs_compose(XsRun r1, XsRun r2) {
    if (r1.e == XS_NO_BINADE) return r2;
    if (r2.e == XS_NO_BINADE) return r1;
    XsRun r;
    r.e = r1.e;
    r.a = r1.a + ((r1.a & 1) ? r2.b : r2.a);
    r.b = r1.b + ((r1.b & 1) ? r2.a : r2.b);
    return r;
}

/* apply a run to a float s that lies in the run's binade */
XS_FN float xs_apply(float s, XsRun r) {
    if (r.e == XS_NO_BINADE) return s;
    uint32_t bits = xs_fbits(s);
    uint32_t M = (bits & 0x7FFFFFu) | 0x800000u;             /* s / u */
    uint32_t k = (uint32_t)((M & 1u) ? r.b : r.a);
    uint32_t M2 = M + k;                                      /* < 2^24 by construction */
    return xs_bitsf(((uint32_t)(r.e + 127) << 23) | (M2 & 0x7FFFFFu));
}

#endif /* EMBER_B200_EXACT_SUM_CORE_H */
