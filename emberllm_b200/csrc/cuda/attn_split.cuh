// attn_split.cuh — decode attention for one position, split over the cache.
//
// The reference (src/model.c:221-259) computes, per query head, the scores of
// positions 0..pos, a softmax whose denominator is ONE sequential fp32 sum over
// t, and outputs that are sequential fp32 sums over t. The scores are
// independent per position, so they spread over many CTAs; the two sequential
// sums are chains whose order is fixed, so they stay one thread per chain.
//
//   attn_scores_kernel     grid (kv heads, ctx / AS_PER). Before its dependency
//                          wait a CTA requests the keys of its AS_PER positions
//                          (one 2-D TMA box [hd][AS_PER] of the transposed cache).
//                          After it, it applies QK-norm and RoPE to this
//                          position's q of the kv head's query heads and to k (the
//                          split-0 CTA stores k and v in the cache), and scores its
//                          positions: one thread per position, the chains of all
//                          query heads side by side (sum_i q_i*k_i in index order,
//                          then * 1/sqrt(hd)). It writes the scores and its
//                          per-head maximum.
//   attn_softmax_pv_kernel grid (kv heads, hd / 32). The maximum over the splits
//                          (order-free), e_t = expf(s_t - max), the denominator as
//                          the reference's sequential sum (one chain per head),
//                          w_t = e_t * (1/den), all in shared memory; then
//                          o_i = sum_t w_t*v_t,i for the CTA's 32 dimensions, one
//                          chain per (head, i), over value slices
//                          [AS_VB positions][32] that a producer thread streams by
//                          TMA while each head's warp consumes them; then the
//                          Q8_0 quantization of each 32-block for the wo matmul.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace emb {

constexpr int AS_THREADS = 256;
constexpr int AS_MAX_KVMUL = 7;     // query heads per kv head (one warp each + one for k)
constexpr int AS_PER = 128;         // cached positions scored per CTA
constexpr int AS_VB = 128;          // positions per value stage
constexpr int AS_VSTAGES = 8;

struct AttnSplitArgs {
    const float *q, *k, *v;        // this position's projections (bias already added)
    void *kc, *vc;                 // this layer's cache: keys [n_kv][hd][kstride], values [n_kv][ctx][hd]
    const float *q_norm, *k_norm;  // QK-norm weights [hd] or NULL
    const float2 *rope;            // [ctx][hd/2] (cos, sin)
    int *ctl;
    float *att;                    // [nh][ast]: scores (written by the scores kernel)
    float *wglob;                  // [n_kv][hd/32][kv_mul][ast]: per-CTA weights when not in smem
    float *pmax;                   // [nh][splits]: per-split maxima of the scores
    int8_t *oq;                    // outputs: Q8 of the head outputs [nh*hd] ...
    float *od;                     //   ... their scales [nh*hd/32]
    float *of;                     //   ... and the fp32 values (may be NULL)
    int nh, nkv, hd, ctx, kstride, neox, splits;
    int ast;                       // att row stride: ctx rounded up to 4 (16-byte rows)
    int w_smem;                    // softmax weights in shared memory (else in att)
    float eps;
    ExpfDev ex;
};

// dynamic shared memory of the two kernels
__host__ __device__ inline size_t as_scores_smem(int hd, int es) { return (size_t)hd * AS_PER * es; }
__host__ __device__ inline size_t as_pv_smem(int kv_mul, int ctx, int es, int w_smem) {
    return (size_t)AS_VSTAGES * AS_VB * 32 * es + (w_smem ? (size_t)kv_mul * ((ctx + 63) / 64 * 64) * 4 : 0);
}

// 2-D TMA load of a box at (x, y) into this CTA only, completing on `bar`
EMB_DEV void as_tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// R: query heads per kv head rounded up to 1, 2, 4 or 8 (register chains)
template <typename T, int R>
__global__ void __launch_bounds__(AS_THREADS) attn_scores_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                 const AttnSplitArgs a) {
    extern __shared__ __align__(128) unsigned char as_smem[];
    __shared__ float qs[R][256];
    __shared__ float ks[256];
    __shared__ float nq_s[256], nk_s[256];
    __shared__ float2 cs_s[128];
    __shared__ float s_scale[R + 1];
    __shared__ float red[R][AS_THREADS / 32];
    __shared__ __align__(8) uint64_t bar;
    T *kbuf = reinterpret_cast<T *>(as_smem);     // [hd][AS_PER]
    const int kvh = blockIdx.x, sp = blockIdx.y, tid = threadIdx.x, hd = a.hd;
    const int kv_mul = a.nh / a.nkv;
    const int warp = tid >> 5, lane = tid & 31;
    int *err = a.ctl + CTL_ERR;
    T *kt = reinterpret_cast<T *>(a.kc) + (size_t)kvh * hd * a.kstride;

    // ---- pre-wait: data of earlier launches only ----
    EMB_PROBE(6, 0);
    const int pos = a.ctl[CTL_POS];
    const int t0 = sp * AS_PER, t1 = min(t0 + AS_PER, pos + 1);
    const int nk = min(t1, pos) - t0;             // cached positions of this split (< pos)
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        if (nk > 0) {
            // keys of positions [t0, t0 + AS_PER) of all hd dimensions; positions
            // at and past pos in the box are not read
            mbar_expect_tx(&bar, (uint32_t)(AS_PER * hd * sizeof(T)));
            as_tma_2d(kbuf, &kmap, t0, kvh * hd, &bar);
        }
    }
    if (tid < hd) {
        nq_s[tid] = a.q_norm ? a.q_norm[tid] : 0.0f;
        nk_s[tid] = a.k_norm ? a.k_norm[tid] : 0.0f;
    }
    if (tid < hd / 2) cs_s[tid] = a.rope[(size_t)pos * (hd / 2) + tid];
    EMB_PROBE(6, 1);
    pdl_wait_then_release();
    EMB_PROBE(6, 2);

    // ---- this position's q (the kv head's query heads) and k ----
    for (int idx = tid; idx < kv_mul * hd; idx += AS_THREADS) {
        const int r = idx / hd, i = idx - r * hd;
        qs[r][i] = a.q[(size_t)(kvh * kv_mul + r) * hd + i];
    }
    if (tid < hd) ks[tid] = a.k[kvh * hd + tid];
    __syncthreads();
    if (a.q_norm) {
        // per-head RMSNorm (ref src/model.c:386-389): one chain per head, one warp each
        if (lane == 0 && warp <= kv_mul) {
            const float *v = warp < kv_mul ? qs[warp] : ks;
            s_scale[warp] = rms_scale(chain_sumsq(v, hd), hd, a.eps);
        }
        __syncthreads();
        for (int idx = tid; idx < (kv_mul + 1) * hd; idx += AS_THREADS) {
            const int r = idx / hd, i = idx - r * hd;
            if (r < kv_mul) qs[r][i] = fmul(fmul(qs[r][i], s_scale[r]), nq_s[i]);
            else ks[i] = fmul(fmul(ks[i], s_scale[kv_mul]), nk_s[i]);
        }
        __syncthreads();
    }
    // RoPE (ref src/model.c:66-80) with the host-built cos/sin table
    for (int idx = tid; idx < (kv_mul + 1) * (hd / 2); idx += AS_THREADS) {
        const int r = idx / (hd / 2), i = idx - r * (hd / 2);
        float *v = r < kv_mul ? qs[r] : ks;
        const int ia = a.neox ? i : 2 * i, ib = a.neox ? i + hd / 2 : 2 * i + 1;
        const float2 cs = cs_s[i];
        const float v0 = v[ia], v1 = v[ib];
        v[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        v[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
    }
    __syncthreads();
    // KV store (ref src/model.c:39-48) by the split-0 CTA; every CTA scores
    // t == pos with the stored (rounded) key
    if (tid < hd) {
        T kq;
        kv_round(ks[tid], &kq);
        if (sp == 0) {
            T vq;
            kv_round(a.v[kvh * hd + tid], &vq);
            kt[(size_t)tid * a.kstride + pos] = kq;
            reinterpret_cast<T *>(a.vc)[((size_t)kvh * a.ctx + pos) * hd + tid] = vq;
        }
        ks[tid] = widen(kq);
    }
    EMB_PROBE(6, 3);
    if (nk > 0) mbar_wait_cta(&bar, 0, err, ERR_ATTN_WAIT);
    else __syncthreads();
    EMB_PROBE(6, 4);

    // ---- scores of this split's positions ----
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    float mloc[R];
#pragma unroll
    for (int r = 0; r < R; r++) mloc[r] = -INFINITY;
    const int t = t0 + tid;
    if (tid < AS_PER && t < t1) {
        float sc[R];
#pragma unroll
        for (int r = 0; r < R; r++) sc[r] = 0.0f;
        if (t == pos) {
            for (int i = 0; i < hd; i++) {
#pragma unroll
                for (int r = 0; r < R; r++) sc[r] = fadd(sc[r], fmul(qs[r][i], ks[i]));
            }
        } else {
            for (int i = 0; i < hd; i += 8) {
                float kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = widen(kbuf[(size_t)(i + j) * AS_PER + tid]);
#pragma unroll
                for (int j = 0; j < 8; j++)
#pragma unroll
                    for (int r = 0; r < R; r++) sc[r] = fadd(sc[r], fmul(qs[r][i + j], kk[j]));
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
            if (r < kv_mul) {
                const float v = fmul(sc[r], inv_sqrt);
                a.att[(size_t)(kvh * kv_mul + r) * a.ast + t] = v;
                mloc[r] = v;
            }
    }
    EMB_PROBE(6, 5);
    // per-head maximum of this split (order-free)
#pragma unroll
    for (int r = 0; r < R; r++) {
        const float m = warp_max(mloc[r]);
        if (lane == 0) red[r][warp] = m;
    }
    __syncthreads();
    if (tid < kv_mul) {
        float m = red[tid][0];
        for (int w = 1; w < AS_THREADS / 32; w++) m = fmaxf(m, red[tid][w]);
        a.pmax[(size_t)(kvh * kv_mul + tid) * a.splits + sp] = m;
    }
    EMB_PROBE(6, 6);
}

// WS: the weights live in shared memory (the compiler then emits shared-memory
// loads for the chains; a pointer that may be either needs generic loads, which
// roughly double the latency each chain step waits on)
template <typename T, bool WS>
__global__ void __launch_bounds__(AS_THREADS) attn_softmax_pv_kernel(const __grid_constant__ CUtensorMap vmap,
                                                                     const AttnSplitArgs a) {
    extern __shared__ __align__(128) unsigned char as_smem[];
    __shared__ float s_max[AS_MAX_KVMUL], s_inv[AS_MAX_KVMUL];
    __shared__ __align__(8) uint64_t full[AS_VSTAGES], cons[AS_VSTAGES];
    __shared__ double tab_s[64];
    const int kvh = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, hd = a.hd;
    const int kv_mul = a.nh / a.nkv;
    const int warp = tid >> 5, lane = tid & 31;
    int *err = a.ctl + CTL_ERR;
    T *vbuf = reinterpret_cast<T *>(as_smem);                                   // [stages][AS_VB][32]
    // weights [kv_mul][ast]: in shared memory when they fit, else in this CTA's own
    // global scratch (the hd/32 CTAs of a kv head each hold a copy)
    float *ws = WS ? reinterpret_cast<float *>(as_smem + (size_t)AS_VSTAGES * AS_VB * 32 * sizeof(T))
                   : a.wglob + ((size_t)kvh * gridDim.y + g) * kv_mul * a.ast;
    const int wst = a.ast;
    constexpr uint32_t STAGE_BYTES = AS_VB * 32 * sizeof(T);
    EMB_PROBE(7, 0);
    const int pos = a.ctl[CTL_POS];
    const int P = pos + 1;
    const int nstage = (P + AS_VB - 1) / AS_VB;
    // pre-wait: value stages entirely before pos (written by earlier steps), the expf table
    if (tid == 0) {
        for (int k = 0; k < AS_VSTAGES; k++) {
            mbar_init(&full[k], 1);
            mbar_init(&cons[k], kv_mul);
        }
        fence_mbar_init();
        for (int k = 0; k < AS_VSTAGES && k < nstage && (k + 1) * AS_VB <= pos; k++) {
            mbar_expect_tx(&full[k], STAGE_BYTES);
            as_tma_2d(vbuf + (size_t)k * AS_VB * 32, &vmap, 32 * g, kvh * a.ctx + k * AS_VB, &full[k]);
        }
    }
    expf_table_load(tab_s, a.ex);
    EMB_PROBE(7, 1);
    pdl_wait_then_release();
    EMB_PROBE(7, 2);
    if (tid == 0) {
        for (int k = 0; k < AS_VSTAGES && k < nstage; k++)
            if (!((k + 1) * AS_VB <= pos)) {
                mbar_expect_tx(&full[k], STAGE_BYTES);
                as_tma_2d(vbuf + (size_t)k * AS_VB * 32, &vmap, 32 * g, kvh * a.ctx + k * AS_VB, &full[k]);
            }
    }

    // the scores of this kv head's query heads
    if (tid < kv_mul) {
        float m = -INFINITY;
        for (int s = 0; s < a.splits; s++) m = fmaxf(m, a.pmax[(size_t)(kvh * kv_mul + tid) * a.splits + s]);
        s_max[tid] = m;
    }
    __syncthreads();
    EMB_PROBE(7, 3);
    // e_t = expf(s_t - max) (ref src/model.c:60): the scores are copied first
    // (all loads in flight), then exponentiated in place
    const float *sc = a.att + (size_t)kvh * kv_mul * a.ast;
    if (WS) {
        const int n4 = kv_mul * (wst / 4);
        const float4 *src = reinterpret_cast<const float4 *>(sc);
        float4 *dst = reinterpret_cast<float4 *>(ws);
        for (int base = 0; base < n4; base += AS_THREADS * 4) {
            float4 v[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (base + j * AS_THREADS + tid < n4) v[j] = src[base + j * AS_THREADS + tid];
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (base + j * AS_THREADS + tid < n4) dst[base + j * AS_THREADS + tid] = v[j];
        }
        __syncthreads();
    }
    // (and zeros up to a multiple of 64 positions: trailing +0 terms leave the
    // sums unchanged; the row stride is a multiple of 64)
    const int Ppad = (P + 63) / 64 * 64;
    for (int r = 0; r < kv_mul; r++) {
        const float mx = s_max[r];
        float *wr = ws + (size_t)r * wst;
        const float *sr = WS ? wr : sc + (size_t)r * a.ast;
        for (int t = tid; t < Ppad; t += AS_THREADS) wr[t] = t < P ? expf_exact(a.ex, tab_s, fsub(sr[t], mx)) : 0.0f;
    }
    __syncthreads();
    EMB_PROBE(7, 4);
    // denominators: the sequential sum over t (ref src/model.c:61), head by head,
    // each by the whole block (split_chain_sum)
#ifdef EMBER_PROBES
    const long long c0 = clock64();
#endif
    for (int r = 0; r < kv_mul; r++) {
        const float den = split_chain_sum<AS_THREADS>(ws + (size_t)r * wst, Ppad);
        if (tid == 0) s_inv[r] = fdiv(1.0f, den);
    }
#ifdef EMBER_PROBES
    if (blockIdx.x == 0 && tid == 0) g_probe[7][10] = (unsigned long long)(clock64() - c0);
#endif
    __syncthreads();
    EMB_PROBE(7, 5);
    for (int r = 0; r < kv_mul; r++) {
        const float inv = s_inv[r];
        for (int t = tid; t < P; t += AS_THREADS) ws[(size_t)r * wst + t] = fmul(ws[(size_t)r * wst + t], inv);
    }
    __syncthreads();
    EMB_PROBE(7, 6);

    // o_i = sum_t w_t * v_t,i in position order (ref src/model.c:252-256): warp r
    // (< kv_mul) carries head r's chains for the CTA's 32 dimensions; the last
    // warp refills each value stage once every head's warp has consumed it
    if (warp < kv_mul) {
        float o = 0.0f;
        const float *w = ws + (size_t)warp * wst;
#ifdef EMBER_PROBES
        unsigned long long wait_ns = 0;
        const long long c1 = clock64();
#endif
        for (int k = 0; k < nstage; k++) {
            const int slot = k % AS_VSTAGES;
            int ok = 1;
#ifdef EMBER_PROBES
            const unsigned long long tw0 = probe_now();
#endif
            if (lane == 0) ok = mbar_wait(&full[slot], (uint32_t)((k / AS_VSTAGES) & 1), err, ERR_ATTN_WAIT);
#ifdef EMBER_PROBES
            wait_ns += probe_now() - tw0;
#endif
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const T *vs = vbuf + (size_t)slot * AS_VB * 32;
            const int n = min(AS_VB, P - k * AS_VB);
            const float *wk = w + k * AS_VB;
            int t = 0;
            if (n >= 16) {
                // products of the next 8 positions are formed while the current 8 are added
                float pa[8], pb[8];
#pragma unroll
                for (int j = 0; j < 8; j++) pa[j] = fmul(wk[j], widen(vs[j * 32 + lane]));
                t = 8;
                for (; t + 16 <= n; t += 16) {
#pragma unroll
                    for (int j = 0; j < 8; j++) pb[j] = fmul(wk[t + j], widen(vs[(t + j) * 32 + lane]));
#pragma unroll
                    for (int j = 0; j < 8; j++) o = fadd(o, pa[j]);
#pragma unroll
                    for (int j = 0; j < 8; j++) pa[j] = fmul(wk[t + 8 + j], widen(vs[(t + 8 + j) * 32 + lane]));
#pragma unroll
                    for (int j = 0; j < 8; j++) o = fadd(o, pb[j]);
                }
                // pa holds positions t-8 .. t-1
#pragma unroll
                for (int j = 0; j < 8; j++) o = fadd(o, pa[j]);
            }
            for (; t < n; t++) o = fadd(o, fmul(wk[t], widen(vs[t * 32 + lane])));
            __syncwarp();
            if (lane == 0) mbar_arrive(&cons[slot]);
        }
        EMB_PROBE(7, 7);
#ifdef EMBER_PROBES
        if (blockIdx.x == 0 && tid == 0) {
            g_probe[7][9] = wait_ns;
            g_probe[7][11] = (unsigned long long)(clock64() - c1);
        }
#endif
        const int gi = (kvh * kv_mul + warp) * hd + g * 32 + lane;
        if (a.of) a.of[gi] = o;
        float dq;
        const int8_t q = quant_lane(o, &dq);
        a.oq[gi] = q;
        if (lane == 0) a.od[gi / 32] = dq;
    } else if (warp == AS_THREADS / 32 - 1 && lane == 0) {
        // producer: stage k + AS_VSTAGES replaces stage k once its consumers are done
        for (int k = 0; k + AS_VSTAGES < nstage; k++) {
            const int slot = k % AS_VSTAGES;
            if (!mbar_wait_backoff(&cons[slot], (uint32_t)((k / AS_VSTAGES) & 1), err, ERR_ATTN_WAIT)) break;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(&full[slot], STAGE_BYTES);
            as_tma_2d(vbuf + (size_t)slot * AS_VB * 32, &vmap, 32 * g, kvh * a.ctx + (k + AS_VSTAGES) * AS_VB,
                      &full[slot]);
        }
    }
    // every value copy has landed before the CTA exits
    if (tid == 0)
        for (int k = nstage - AS_VSTAGES < 0 ? 0 : nstage - AS_VSTAGES; k < nstage; k++)
            mbar_wait(&full[k % AS_VSTAGES], (uint32_t)((k / AS_VSTAGES) & 1), err, ERR_ATTN_WAIT);
}

}  // namespace emb
