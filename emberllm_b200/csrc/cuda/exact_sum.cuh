// exact_sum.cuh — the sequential fp32 sum of non-negative terms, evaluated by a
// whole CTA in parallel with a bit-identical result (exact_sum_core.h explains
// why this is possible). Phases, for NT threads each owning M = ceil(n/NT)
// consecutive terms:
//   A/B  double-precision prefix of the terms (per-thread sums, warp shuffles,
//        a scan of the warp totals): the exact prefix sum to ~1e-13;
//   C    each thread classifies its steps: a step whose running sum stays in one
//        certain binade becomes a pair (run step), the others stay float adds;
//        consecutive run steps are composed;
//   D    a segmented scan of (has-a-float-add, open run) over the threads gives
//        each thread the run that enters it; a scan of item counts gives offsets;
//   E    threads write their items (runs and float adds) in global order;
//   F    one thread applies the items in order (typically a few dozen).
// If the item list would overflow, one thread falls back to the plain chain.
#pragma once

#include "common.cuh"
#include "exact_sum_core.h"

namespace emb {

constexpr int XS_MAX_ITEMS = 256;

struct XsItem {
    int step;   // 1: float add of p; 0: run (e, a, b)
    int e, a, b;
    float p;
};

struct XsScratch {
    double wsum[32];
    int wflag[32], we[32], wa[32], wb[32], wcnt[32];
    float result;
    int total;
    XsItem items[XS_MAX_ITEMS];
};

EMB_DEV void xs_seg(int &f, XsRun &r, int f2, XsRun r2) {
    r = f2 ? r2 : xs_compose(r, r2);
    f |= f2;
}

// Classify and fold the steps [i0, i1) of one thread, whose running sums start
// at the exact prefix D. Pass 1 (emit == false) returns the summary; pass 2
// writes the items, the first run prefixed by `carry`.
EMB_DEV void xs_fold(const float *v, int i0, int i1, double D, bool emit, XsRun carry, XsItem *out,
                     int &flag, XsRun &cur, int &count) {
    flag = 0;
    count = 0;
    cur = xs_empty();
    int w = 0;
    for (int i = i0; i < i1; i++) {
        const float p = v[i];
        const double Dn = __dadd_rn(D, (double)p);
        const int e0 = xs_certain_binade(D, i), e1 = xs_certain_binade(Dn, i + 1);
        if (e0 != XS_NO_BINADE && e0 == e1) {
            XsRun st;
            st.e = e0;
            xs_step_pair(p, e0, &st.a, &st.b);
            cur = xs_compose(cur, st);
        } else {
            if (!flag) {
                if (emit) { XsRun r = xs_compose(carry, cur); out[w++] = XsItem{0, r.e, r.a, r.b, 0.0f}; }
                count = 1;
            } else if (cur.e != XS_NO_BINADE) {
                if (emit) out[w++] = XsItem{0, cur.e, cur.a, cur.b, 0.0f};
                count++;
            }
            if (emit) out[w++] = XsItem{1, 0, 0, 0, p};
            count++;
            flag = 1;
            cur = xs_empty();
        }
        D = Dn;
    }
}

// sum = ((0 + v[0]) + v[1]) + ... + v[n-1] for v[i] >= 0 (finite), every thread
// of the CTA (NT threads) must call it; the result is returned to all.
template <int NT>
__device__ float exact_pos_sum(const float *v, int n, XsScratch *sc) {
    constexpr unsigned FULL = 0xffffffffu;
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = (n + NT - 1) / NT;
    const int i0 = min(tid * M, n), i1 = min(i0 + M, n);

    // A/B: exclusive double prefix of the terms
    double T = 0.0;
    for (int i = i0; i < i1; i++) T = __dadd_rn(T, (double)v[i]);
    double inc = T;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double y = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc = __dadd_rn(inc, y);
    }
    double ex = __shfl_up_sync(FULL, inc, 1);
    if (lane == 0) ex = 0.0;
    if (lane == 31) sc->wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        double w = lane < NW ? sc->wsum[lane] : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double y = __shfl_up_sync(FULL, w, o);
            if (lane >= o) w = __dadd_rn(w, y);
        }
        double wex = __shfl_up_sync(FULL, w, 1);
        if (lane == 0) wex = 0.0;
        __syncwarp();
        if (lane < NW) sc->wsum[lane] = wex;
    }
    __syncthreads();
    const double base = __dadd_rn(sc->wsum[warp], ex);

    // C: summary of this thread's steps
    int flag, cnt;
    XsRun run;
    xs_fold(v, i0, i1, base, false, xs_empty(), nullptr, flag, run, cnt);

    // D: segmented scan of (flag, run), scan of counts
    int f_in = flag, c_in = cnt;
    XsRun r_in = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int f2 = __shfl_up_sync(FULL, f_in, o), c2 = __shfl_up_sync(FULL, c_in, o);
        XsRun r2;
        r2.e = __shfl_up_sync(FULL, r_in.e, o);
        r2.a = __shfl_up_sync(FULL, r_in.a, o);
        r2.b = __shfl_up_sync(FULL, r_in.b, o);
        if (lane >= o) {
            // (earlier) ⊕ (mine)
            int f = f2;
            XsRun r = r2;
            xs_seg(f, r, f_in, r_in);
            f_in = f;
            r_in = r;
            c_in += c2;
        }
    }
    // exclusive within the warp
    int f_ex = __shfl_up_sync(FULL, f_in, 1), c_ex = __shfl_up_sync(FULL, c_in, 1);
    XsRun r_ex;
    r_ex.e = __shfl_up_sync(FULL, r_in.e, 1);
    r_ex.a = __shfl_up_sync(FULL, r_in.a, 1);
    r_ex.b = __shfl_up_sync(FULL, r_in.b, 1);
    if (lane == 0) { f_ex = 0; c_ex = 0; r_ex = xs_empty(); }
    if (lane == 31) {
        sc->wflag[warp] = f_in; sc->we[warp] = r_in.e; sc->wa[warp] = r_in.a; sc->wb[warp] = r_in.b;
        sc->wcnt[warp] = c_in;
    }
    __syncthreads();
    if (tid == 0) {
        // exclusive scan of the warp totals, in place (NW <= 32 values, sequential)
        int f = 0, c = 0;
        XsRun r = xs_empty();
        for (int w = 0; w < NW; w++) {
            int fw = sc->wflag[w], cw = sc->wcnt[w];
            XsRun rw;
            rw.e = sc->we[w]; rw.a = sc->wa[w]; rw.b = sc->wb[w];
            sc->wflag[w] = f; sc->we[w] = r.e; sc->wa[w] = r.a; sc->wb[w] = r.b; sc->wcnt[w] = c;
            xs_seg(f, r, fw, rw);
            c += cw;
        }
    }
    __syncthreads();
    int f_carry = sc->wflag[warp];
    XsRun carry;
    carry.e = sc->we[warp]; carry.a = sc->wa[warp]; carry.b = sc->wb[warp];
    xs_seg(f_carry, carry, f_ex, r_ex);                 // run entering this thread
    const int offset = sc->wcnt[warp] + c_ex;
    if (tid == NT - 1) {
        const int total = offset + cnt + 1;
        sc->total = total;
        if (total <= XS_MAX_ITEMS) {
            int f = f_carry;
            XsRun r = carry;
            xs_seg(f, r, flag, run);                    // the final open run
            sc->items[total - 1] = XsItem{0, r.e, r.a, r.b, 0.0f};
        }
    }
    __syncthreads();
    const int total = sc->total;
    // E: items in order
    if (total <= XS_MAX_ITEMS && flag) {
        int f2, c2;
        XsRun r2;
        xs_fold(v, i0, i1, base, true, carry, sc->items + offset, f2, r2, c2);
    }
    __syncthreads();
    // F: apply
    if (tid == 0) {
        float s = 0.0f;
        if (total <= XS_MAX_ITEMS) {
            for (int k = 0; k < total; k++) {
                const XsItem it = sc->items[k];
                if (it.step) s = __fadd_rn(s, it.p);
                else { XsRun r; r.e = it.e; r.a = it.a; r.b = it.b; s = xs_apply(s, r); }
            }
        } else {
            s = chain_sum(0.0f, v, n);
        }
        sc->result = s;
    }
    __syncthreads();
    return sc->result;
}

}  // namespace emb
