/* exact_sum_check.c — host check of the parallel exact sum (csrc/exact_sum_core.h).
 *
 * Emulates, thread by thread, the phases the device function runs in a CTA of NT
 * threads (double prefix scan, per-thread run folding, segmented scan of runs,
 * item emission, in-order application) and compares the result bit for bit
 * with the plain sequential float sum, over many vectors drawn from
 * distributions chosen to hit ties, binade crossings, zeros, tiny and huge terms.
 * Build: gcc -O2 -fno-fast-math -ffp-contract=off -I<csrc> exact_sum_check.c
 * Prints "ok <count>" or the first mismatch.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "exact_sum_core.h"

#define NT 256
#define MAX_ITEMS 512

typedef struct { int step; float p; XsRun r; } Item;

static float serial(const float *v, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += v[i];
    return s;
}

/* returns the emulated CTA result; *fallback set when the item list overflowed */
static float parallel(const float *v, int n, int *fallback, int *nitems_out) {
    static double T[NT], base[NT];
    static int flag[NT], cnt[NT], off[NT];
    static XsRun sum_run[NT], carry[NT];
    static Item items[MAX_ITEMS + NT * 64];
    const int M = (n + NT - 1) / NT;
    /* A: local double sums;  B: exclusive prefix (order of the device's scan is
       irrelevant for the bounds: any double summation order errs by ~1e-13) */
    for (int t = 0; t < NT; t++) {
        int i0 = t * M < n ? t * M : n, i1 = i0 + M < n ? i0 + M : n;
        T[t] = 0;
        for (int i = i0; i < i1; i++) T[t] += (double)v[i];
    }
    double acc = 0;
    for (int t = 0; t < NT; t++) { base[t] = acc; acc += T[t]; }
    /* C: pass 1 per thread */
    for (int t = 0; t < NT; t++) {
        int i0 = t * M < n ? t * M : n, i1 = i0 + M < n ? i0 + M : n;
        double D = base[t];
        XsRun pre = xs_empty(), cur = xs_empty();
        int has = 0, c = 0;
        for (int i = i0; i < i1; i++) {
            double Dn = D + (double)v[i];
            int e0 = xs_certain_binade(D, i), e1 = xs_certain_binade(Dn, i + 1);
            if (e0 != XS_NO_BINADE && e0 == e1) {
                XsRun st; st.e = e0;
                xs_step_pair(v[i], e0, &st.a, &st.b);
                cur = xs_compose(cur, st);
            } else {
                if (!has) { pre = cur; c = 1; }
                else if (cur.e != XS_NO_BINADE) c++;
                c++;
                has = 1;
                cur = xs_empty();
            }
            D = Dn;
        }
        flag[t] = has;
        sum_run[t] = cur;            /* the suffix run, or the whole chunk's run */
        cnt[t] = c;
        (void)pre;
    }
    /* D: segmented exclusive scan of (flag, run); exclusive scan of counts */
    XsRun r = xs_empty();
    int o = 0;
    for (int t = 0; t < NT; t++) {
        carry[t] = r;
        off[t] = o;
        r = flag[t] ? sum_run[t] : xs_compose(r, sum_run[t]);
        o += cnt[t];
    }
    int total = o + 1;
    *nitems_out = total;
    if (total > MAX_ITEMS) { *fallback = 1; return serial(v, n); }
    *fallback = 0;
    /* E: pass 2 emission */
    for (int t = 0; t < NT; t++) {
        if (!flag[t]) continue;
        int i0 = t * M < n ? t * M : n, i1 = i0 + M < n ? i0 + M : n;
        double D = base[t];
        XsRun cur = xs_empty();
        int first = 1, w = off[t];
        for (int i = i0; i < i1; i++) {
            double Dn = D + (double)v[i];
            int e0 = xs_certain_binade(D, i), e1 = xs_certain_binade(Dn, i + 1);
            if (e0 != XS_NO_BINADE && e0 == e1) {
                XsRun st; st.e = e0;
                xs_step_pair(v[i], e0, &st.a, &st.b);
                cur = xs_compose(cur, st);
            } else {
                if (first) { items[w].step = 0; items[w].r = xs_compose(carry[t], cur); w++; first = 0; }
                else if (cur.e != XS_NO_BINADE) { items[w].step = 0; items[w].r = cur; w++; }
                items[w].step = 1; items[w].p = v[i]; w++;
                cur = xs_empty();
            }
            D = Dn;
        }
    }
    items[total - 1].step = 0;
    items[total - 1].r = r;          /* the final open run */
    /* F: in-order application */
    float s = 0.0f;
    for (int k = 0; k < total; k++) s = items[k].step ? s + items[k].p : xs_apply(s, items[k].r);
    return s;
}

static unsigned long long rs = 88172645463325252ull;
static double urand(void) { rs ^= rs << 13; rs ^= rs >> 7; rs ^= rs << 17; return (rs >> 11) * 0x1p-53; }
static double nrand(void) { double u = urand() + 1e-300, w = urand(); return sqrt(-2 * log(u)) * cos(6.283185307179586 * w); }

int main(int argc, char **argv) {
    int iters = argc > 1 ? atoi(argv[1]) : 20000;
    static float v[8192];
    long checked = 0, fallbacks = 0, maxitems = 0;
    for (int it = 0; it < iters; it++) {
        int kind = it % 11;
        int n = 1 + (int)(urand() * (kind < 3 ? 1024 : (kind < 6 ? 300 : 8192)));
        double sc = pow(10.0, urand() * 8 - 4);
        for (int i = 0; i < n; i++) {
            double x;
            switch (kind) {
            case 0: x = nrand() * sc; x = (float)x * (float)x; break;          /* RMSNorm squares */
            case 1: x = exp(-urand() * 20); break;                               /* softmax terms */
            case 2: x = (urand() < 0.3) ? 0.0 : ldexp(1.0, (int)(urand() * 20) - 10); break; /* powers of two: ties */
            case 3: x = (double)((int)(urand() * 8)) * 0.125; break;             /* few bits: many ties */
            case 4: x = i == 0 ? 0.0 : urand() * sc; break;                      /* leading zero */
            case 5: x = urand() < 0.01 ? 1e6 * sc : urand() * sc; break;         /* spikes */
            case 6: x = 1.0; break;                                              /* equal terms */
            case 7: x = ldexp(urand(), -(int)(urand() * 40)); break;             /* wide range */
            case 8: x = (float)(nrand() * 0.5) * (float)(nrand() * 0.5); x = x < 0 ? -x : x; break;
            case 9: x = i == 0 ? 16777216.0 : (urand() < 0.5 ? 1.0 : 3.0); break;  /* half-ulp ties */
            default: x = i == 0 ? ldexp(1.0, 20) : ldexp(1.0, -4 + (int)(urand() * 3)); break;
            }
            v[i] = (float)x;
        }
        int fb = 0, ni = 0;
        float a = serial(v, n), b = parallel(v, n, &fb, &ni);
        fallbacks += fb;
        if (ni > maxitems) maxitems = ni;
        if (xs_fbits(a) != xs_fbits(b)) {
            printf("MISMATCH kind %d n %d serial %a parallel %a\n", kind, n, a, b);
            return 1;
        }
        checked++;
    }
    printf("ok %ld fallbacks %ld max_items %ld\n", checked, fallbacks, maxitems);
    return 0;
}
