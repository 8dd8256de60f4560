// attn_decode.cuh — decode attention of one query position per (head [, stream])
// (ref src/model.c:221-259): the single-token step's kernel and, as a template
// mode, the batched decode of independent streams. Templates only, so both the
// token-step and the batched-pipeline translation units include it.
#pragma once

#include "common.cuh"

namespace emb {

constexpr int ATTN_THREADS = 256;

// ---------------------------------------------------------------- attention ----

struct AttnArgs {
    const float *q, *k, *v;        // this position's projections (bias already added)
    void *kc;                      // this layer's keys, transposed: [n_kv][hd][kstride]
    void *vc;                      // this layer's values: [n_kv][ctx][hd]
    const float *q_norm, *k_norm;  // QK-norm weights [hd] or NULL
    const float2 *rope;            // [ctx][hd/2] (cos, sin)
    int *ctl;
    float *att;                    // global scores [n_heads][ctx] when they do not fit smem
    int8_t *oq;                    // outputs: Q8 of the head outputs [n_heads*hd] ...
    float *od;                     //   ... their scales [n_heads*hd/32]
    float *of;                     //   ... and the fp32 values (may be NULL)
    int nh, nkv, hd, ctx, kstride, neox, att_in_smem;
    int chunk;                     // cached positions per staged chunk
    float eps;
    ExpfDev ex;
    // batched decode of independent streams (BATCH: one CTA per (head, stream)):
    // stream t's position bpos[t], its cache at kc/vc + t * cache_stride
    // elements, its roped query at q + t * nh * hd (the cache already holds its
    // key and value), outputs into the token-row GEMM layout
    const int *bpos;
    size_t cache_stride;
    int8_t *bxq;                   // [n_pad][k_pad]
    float *bxs;                    // [nh*hd/32][n_pad]
    int k_pad, n_pad;
};


// Copy keys of positions [c0, c0+n) (all hd rows of the transposed layout) into
// kbuf[hd][CH] with 16-byte asynchronous copies by all threads. Rows are padded
// to kstride, so rounding n up to a vector stays in bounds; positions from n on
// (the current one included, which this launch writes) are copied but not read.
template <typename T>
EMB_DEV void load_k_chunk(T *kbuf, const T *kt, int kstride, int c0, int n, int hd, int CH) {
    // 16-byte cp.async copies, all in flight at once; the caller waits
    // (cp_async_wait_all + __syncthreads) before reading kbuf
    constexpr int E = 16 / (int)sizeof(T);
    const int nv = (n + E - 1) / E;
    const int total = hd * nv;
    for (int idx = threadIdx.x; idx < total; idx += ATTN_THREADS) {
        const int i = idx / nv, vv = idx - i * nv;
        cp_async16(kbuf + (size_t)i * CH + vv * E, kt + (size_t)i * kstride + c0 + vv * E);
    }
    cp_async_commit();
}

// One query position over the cache for one head (ref src/model.c:221-259).
//
// Pre-wait (data of earlier launches only): the position word, the QK-norm
// weights, this position's cos/sin, the first chunk of cached keys (thread
// loads into a transposed [hd][chunk] buffer) and values (one bulk copy into a
// [chunk][hd] buffer). Post-wait: this position's q/k/v from the projection,
// QK-norm and RoPE, the KV store, then
//   scores  one thread per cached position: sum_i q_i*k_i in index order;
//   softmax max (order-free), expf, the sequential sum, the reciprocal;
//   output  one thread per dimension: sum_t w_t*v_t in position order,
// each chain reading shared memory with its loads batched ahead of the adds.
// Further value chunks ping-pong between the two buffers by bulk copies.
//
// BATCH: one CTA per (query head, stream) of a batched decode step: the query is
// already normed and roped and this position's key and value are in the cache
// (pf_qkv_post_kernel), so the cached positions run 0..pos inclusive; the same
// chains in the same order.
template <typename T, bool BATCH = false>
__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float qs[256], ks[256], vs[256], qn_s[256], kn_s[256];
    __shared__ float2 cs_s[128];
    __shared__ float red[ATTN_THREADS / 32];
    __shared__ float s_q, s_k, s_inv;
    __shared__ double tab_s[64];
    const int h = blockIdx.x, tid = threadIdx.x, hd = a.hd, CH = a.chunk;
    const int kv_mul = a.nh / a.nkv, kvh = h / kv_mul;
    const int warp = tid >> 5, lane = tid & 31;
    const size_t buf_elems = (size_t)CH * hd;
    T *buf0 = reinterpret_cast<T *>(smem);
    T *buf1 = buf0 + buf_elems;
    float *att = a.att_in_smem ? reinterpret_cast<float *>(smem + 2 * buf_elems * sizeof(T))
                               : a.att + (size_t)h * a.ctx;
    int *err = a.ctl + CTL_ERR;
    uint32_t ph0 = 0, ph1 = 0;
    EMB_PROBE(4, 0);

    // ---- pre-wait ----
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    const int bt = BATCH ? (int)blockIdx.y : 0;
    // written by the host or the previous step's tail; BATCH: this stream's
    const int pos = BATCH ? a.bpos[bt] : a.ctl[CTL_POS];
    const int ncache = BATCH ? pos + 1 : pos;   // positions read from the cache
    const size_t coff = BATCH ? (size_t)bt * a.cache_stride : 0;
    T *kt = reinterpret_cast<T *>(a.kc) + coff + (size_t)kvh * hd * a.kstride;
    T *vt = reinterpret_cast<T *>(a.vc) + coff + (size_t)kvh * a.ctx * hd;
    if (!BATCH) {
        if (tid < hd) {
            qn_s[tid] = a.q_norm ? a.q_norm[tid] : 0.0f;
            kn_s[tid] = a.k_norm ? a.k_norm[tid] : 0.0f;
        }
        if (tid < hd / 2) cs_s[tid] = a.rope[(size_t)pos * (hd / 2) + tid];
    }
    expf_table_load(tab_s, a.ex);
    __syncthreads();
    const int nchunks = (ncache + CH - 1) / CH;
    const int n0 = min(CH, ncache);
    if (tid == 0 && n0 > 0) {         // values of chunk 0 -> buf1
        mbar_expect_tx(&bars[1], (uint32_t)(n0 * hd * (int)sizeof(T)));
        bulk_g2s(buf1, vt, (uint32_t)(n0 * hd * sizeof(T)), &bars[1]);
    }
    if (n0 > 0) load_k_chunk(buf0, kt, a.kstride, 0, n0, hd, CH);   // keys of chunk 0 -> buf0 (async)
    EMB_PROBE(4, 1);
    pdl_wait_then_release();
    EMB_PROBE(4, 2);

    if constexpr (BATCH) {
        if (tid < hd) qs[tid] = a.q[(size_t)bt * a.nh * hd + h * hd + tid];
    } else {
        // ---- this position: q, k, v; QK-norm; RoPE; KV store ----
        if (tid < hd) {
            qs[tid] = a.q[h * hd + tid];
            ks[tid] = a.k[kvh * hd + tid];
            vs[tid] = a.v[kvh * hd + tid];
        }
        __syncthreads();
        EMB_PROBE(4, 3);
        if (a.q_norm) {
            // per-head RMSNorm of q and k (ref src/model.c:386-389); the two
            // sequential sums run on different warps
            if (tid == 0) s_q = rms_scale(chain_sumsq(qs, hd), hd, a.eps);
            else if (tid == 32) s_k = rms_scale(chain_sumsq(ks, hd), hd, a.eps);
            __syncthreads();
        }
        EMB_PROBE(4, 4);
        // RoPE (ref src/model.c:66-80) with the host-built cos/sin table; the
        // thread that rotates a pair first applies the QK-norm scale and weights
        // to it, (v*scale)*w, in registers
        if (tid < hd / 2) {
            const int ia = a.neox ? tid : 2 * tid, ib = a.neox ? tid + hd / 2 : 2 * tid + 1;
            const float2 cs = cs_s[tid];
            float q0 = qs[ia], q1 = qs[ib], k0 = ks[ia], k1 = ks[ib];
            if (a.q_norm) {
                q0 = fmul(fmul(q0, s_q), qn_s[ia]);
                q1 = fmul(fmul(q1, s_q), qn_s[ib]);
                k0 = fmul(fmul(k0, s_k), kn_s[ia]);
                k1 = fmul(fmul(k1, s_k), kn_s[ib]);
            }
            qs[ia] = fsub(fmul(q0, cs.x), fmul(q1, cs.y));
            qs[ib] = fadd(fmul(q0, cs.y), fmul(q1, cs.x));
            ks[ia] = fsub(fmul(k0, cs.x), fmul(k1, cs.y));
            ks[ib] = fadd(fmul(k0, cs.y), fmul(k1, cs.x));
        }
        __syncthreads();
        // KV store (ref src/model.c:39-48): the cache holds fp32 or RNE fp16, and
        // attention reads the stored values, including at t == pos
        if (tid < hd) {
            T kq, vq;
            kv_round(ks[tid], &kq);
            kv_round(vs[tid], &vq);
            ks[tid] = widen(kq);
            vs[tid] = widen(vq);
            if (h % kv_mul == 0) {
                kt[(size_t)tid * a.kstride + pos] = kq;
                vt[(size_t)pos * hd + tid] = vq;
            }
        }
    }
    cp_async_wait_all();   // the keys of chunk 0, copied since before the wait
    __syncthreads();

    EMB_PROBE(4, 5);
    // ---- scores: sc = sum_i q_i*k_i in index order, then * (1/sqrt(hd)) ----
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    float lmax = -INFINITY;   // the largest of this thread's scores (the max is order-free)
    for (int c = 0; c < nchunks; c++) {
        const int c0 = c * CH, n = min(CH, ncache - c0);
        if (c > 0) {
            __syncthreads();
            load_k_chunk(buf0, kt, a.kstride, c0, n, hd, CH);
            cp_async_wait_all();
            __syncthreads();
        }
        for (int t = tid; t < n; t += ATTN_THREADS) {
            float sc = 0.0f;
            for (int i = 0; i < hd; i += 8) {
                float kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = widen(buf0[(size_t)(i + j) * CH + t]);
#pragma unroll
                for (int j = 0; j < 8; j++) sc = fadd(sc, fmul(qs[i + j], kk[j]));
            }
            const float s = fmul(sc, inv_sqrt);
            att[c0 + t] = s;
            lmax = fmaxf(lmax, s);
        }
    }
    // the score at t == pos (keys in registers' smem copy), on a thread that had
    // no position in the last chunk
    const int last_n = nchunks > 0 ? pos - (nchunks - 1) * CH : 0;
    if (!BATCH && tid == last_n % ATTN_THREADS) {
        float sc = 0.0f;
        for (int i = 0; i < hd; i++) sc = fadd(sc, fmul(qs[i], ks[i]));
        att[pos] = fmul(sc, inv_sqrt);
        lmax = fmaxf(lmax, att[pos]);
    }
    // ---- softmax (ref src/model.c:57-64): the max is order-free, so each warp
    // reduces its threads' maxima and one barrier publishes them (and the scores)
    lmax = warp_max(lmax);
    if (lane == 0) red[warp] = lmax;
    __syncthreads();
    EMB_PROBE(4, 6);
    // the keys are done: value chunk 1 may stream into buf0 during the softmax
    if (tid == 0 && nchunks > 1) {
        const int n1 = min(CH, ncache - CH);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bars[0], (uint32_t)(n1 * hd * (int)sizeof(T)));
        bulk_g2s(buf0, vt + (size_t)CH * hd, (uint32_t)(n1 * hd * sizeof(T)), &bars[0]);
    }

    float mx = red[0];
#pragma unroll
    for (int w = 1; w < ATTN_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
    EMB_PROBE(4, 10);
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = expf_exact(a.ex, tab_s, fsub(att[t], mx));
    __syncthreads();
    EMB_PROBE(4, 11);
    // the denominator: the reference's sequential sum over t = 0..pos
    if (tid == 0) s_inv = fdiv(1.0f, chain_sum_pipe(0.0f, att, pos + 1));
    __syncthreads();
    EMB_PROBE(4, 12);
    const float inv = s_inv;
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = fmul(att[t], inv);
    __syncthreads();

    EMB_PROBE(4, 7);
    // ---- out_i = sum_t w_t * v_t,i, sequential over t (ref src/model.c:252-256) ----
    float o = 0.0f;
    for (int c = 0; c < nchunks; c++) {
        const int c0 = c * CH, n = min(CH, ncache - c0);
        const bool in1 = (c & 1) == 0;           // chunks 0,2,4.. in buf1; 1,3,.. in buf0
        T *vb = in1 ? buf1 : buf0;
        if (in1) { mbar_wait_cta(&bars[1], ph1, err, ERR_ATTN_WAIT); ph1 ^= 1; }
        else     { mbar_wait_cta(&bars[0], ph0, err, ERR_ATTN_WAIT); ph0 ^= 1; }
        if (tid < hd) {
            const float *w = att + c0;
            int t = 0;
            for (; t + 8 <= n; t += 8) {
                float ww[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) { ww[j] = w[t + j]; vv[j] = widen(vb[(size_t)(t + j) * hd + tid]); }
#pragma unroll
                for (int j = 0; j < 8; j++) o = fadd(o, fmul(ww[j], vv[j]));
            }
            for (; t < n; t++) o = fadd(o, fmul(w[t], widen(vb[(size_t)t * hd + tid])));
        }
        __syncthreads();
        if (tid == 0 && c + 2 < nchunks) {       // refill the freed buffer with chunk c+2
            const int n2 = min(CH, ncache - (c + 2) * CH);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            uint64_t *bb = in1 ? &bars[1] : &bars[0];
            mbar_expect_tx(bb, (uint32_t)(n2 * hd * (int)sizeof(T)));
            bulk_g2s(vb, vt + (size_t)(c + 2) * CH * hd, (uint32_t)(n2 * hd * sizeof(T)), bb);
        }
    }
    EMB_PROBE(4, 8);
    if (tid < hd) {
        if (!BATCH) o = fadd(o, fmul(att[pos], vs[tid]));
        const int gi = h * hd + tid;
        float dq;
        int8_t q = quant_lane(o, &dq);   // hd % 32 == 0: each warp owns one block
        if (BATCH) {
            a.bxq[(size_t)bt * a.k_pad + gi] = q;
            if (lane == 0) a.bxs[(size_t)(gi / 32) * a.n_pad + bt] = dq;
        } else {
            if (a.of) a.of[gi] = o;
            a.oq[gi] = q;
            if (lane == 0) a.od[gi / 32] = dq;
        }
    }
    EMB_PROBE(4, 9);
}

// ---- batched decode: one CTA per (kv head, stream) -----------------------------

constexpr int AB_CH = 64;   // cached positions per staged chunk

// keys of positions [c0, c0+n) -> buf[hd][AB_CH] (the cache keeps keys transposed,
// [hd][kstride]); values -> buf[AB_CH][hd]. 16-byte cp.async by every thread, one
// committed group. Rows are padded to kstride (a multiple of 8) and c0 is a
// multiple of 8, so whole vectors stay in bounds.
template <typename T>
EMB_DEV void ab_stage_k(T *buf, const T *kt, int kstride, int c0, int n, int hd) {
    constexpr int E = 16 / (int)sizeof(T);
    const int nv = (n + E - 1) / E, total = hd * nv;
    for (int idx = threadIdx.x; idx < total; idx += ATTN_THREADS) {
        const int i = idx / nv, v = idx - i * nv;
        cp_async16(buf + (size_t)i * AB_CH + v * E, kt + (size_t)i * kstride + c0 + v * E);
    }
    cp_async_commit();
}
template <typename T>
EMB_DEV void ab_stage_v(T *buf, const T *vt, int c0, int n, int hd) {
    constexpr int E = 16 / (int)sizeof(T);
    const int total = n * hd / E;
    for (int idx = threadIdx.x; idx < total; idx += ATTN_THREADS)
        cp_async16(buf + (size_t)idx * E, vt + (size_t)c0 * hd + (size_t)idx * E);
    cp_async_commit();
}

// dynamic shared memory: two chunk buffers, then the scores [KVM][att_stride]
__host__ inline size_t ab_smem_bytes(int hd, int es, int kvm, int att_stride) {
    return 2 * (size_t)AB_CH * hd * es + (size_t)kvm * att_stride * 4;
}

// One CTA per (kv head, stream) of a batched decode step: the KVM query heads of
// the kv head share every staged chunk of the stream's cache (ref
// src/model.c:221-259, the single-token step's chains in its order):
//   scores   thread (position of the chunk, head): sum_i q_i*k_i in index order;
//   softmax  per head: the max (order-free: each thread keeps its own, a warp
//            reduction, one barrier), expf, the sequential denominator (one
//            lane per head), w = e * (1/den);
//   output   thread (head, dimension): sum_t w_t*v_t in position order, then Q8
//            into the token-row GEMM layout.
// The query is already normed and roped and this position's key and value are
// in the cache (pf_qkv_post_kernel). Key chunks, then value chunks, are
// double-buffered: chunk c+1's copies run while chunk c is used. Needs
// KVM * AB_CH <= 256 and KVM * hd <= 256.
template <typename T, int KVM>
__global__ void __launch_bounds__(ATTN_THREADS) attn_batch_kernel(const AttnArgs a) {
    static_assert(KVM >= 1 && KVM * AB_CH <= ATTN_THREADS, "attn_batch_kernel: KVM * AB_CH <= 256");
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) float qs[256 * KVM];   // [hd][KVM]
    __shared__ float red[ATTN_THREADS / 32];
    __shared__ float s_inv[KVM];
    __shared__ double tab_s[64];
    const int kvh = blockIdx.x, bt = blockIdx.y, tid = threadIdx.x, hd = a.hd;
    const int warp = tid >> 5, lane = tid & 31;
    const int pos = a.bpos[bt], npos = pos + 1;
    const int astr = a.ctx;   // scores row stride (positions)
    const size_t coff = (size_t)bt * a.cache_stride;
    const T *kt = reinterpret_cast<const T *>(a.kc) + coff + (size_t)kvh * hd * a.kstride;
    const T *vt = reinterpret_cast<const T *>(a.vc) + coff + (size_t)kvh * a.ctx * hd;
    T *buf0 = reinterpret_cast<T *>(smem);
    const size_t cbuf = (size_t)AB_CH * hd;
    float *att = reinterpret_cast<float *>(smem + 2 * cbuf * sizeof(T));
    const int nch = (npos + AB_CH - 1) / AB_CH;
    ab_stage_k(buf0, kt, a.kstride, 0, min(AB_CH, npos), hd);
    expf_table_load(tab_s, a.ex);
    for (int idx = tid; idx < KVM * hd; idx += ATTN_THREADS) {
        const int hh = idx / hd, i = idx - hh * hd;
        qs[i * KVM + hh] = a.q[(size_t)bt * a.nh * hd + (size_t)(kvh * KVM + hh) * hd + i];
    }

    // ---- scores: thread (tl, hs) = (position in the chunk, head) ----
    const int tl = tid % AB_CH, hs = tid / AB_CH;
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    float lmax = -INFINITY;
    for (int c = 0; c < nch; c++) {
        const int c0 = c * AB_CH, n = min(AB_CH, npos - c0);
        if (c + 1 < nch) {
            ab_stage_k(buf0 + ((c + 1) & 1) * cbuf, kt, a.kstride, c0 + AB_CH, min(AB_CH, npos - c0 - AB_CH), hd);
            cp_async_wait_1();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const T *kb = buf0 + (c & 1) * cbuf;
        if (hs < KVM && tl < n) {
            float sc = 0.0f;
            for (int i = 0; i < hd; i += 8) {
                float kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = widen(kb[(size_t)(i + j) * AB_CH + tl]);
#pragma unroll
                for (int j = 0; j < 8; j++) sc = fadd(sc, fmul(qs[(i + j) * KVM + hs], kk[j]));
            }
            const float v = fmul(sc, inv_sqrt);
            att[(size_t)hs * astr + c0 + tl] = v;
            lmax = fmaxf(lmax, v);
        }
        __syncthreads();   // the buffer is free for chunk c + 2
    }
    // the first value chunk streams in during the softmax
    ab_stage_v(buf0, vt, 0, min(AB_CH, npos), hd);

    // ---- softmax per head (ref src/model.c:57-64) ----
    // warp w holds positions of head (32 w) / AB_CH: AB_CH / 32 warps per head
    lmax = warp_max(lmax);
    if (lane == 0) red[warp] = lmax;
    __syncthreads();
    float mx[KVM];
#pragma unroll
    for (int hh = 0; hh < KVM; hh++) {
        mx[hh] = red[hh * (AB_CH / 32)];
#pragma unroll
        for (int w = 1; w < AB_CH / 32; w++) mx[hh] = fmaxf(mx[hh], red[hh * (AB_CH / 32) + w]);
    }
#pragma unroll
    for (int hh = 0; hh < KVM; hh++)
        for (int t = tid; t < npos; t += ATTN_THREADS)
            att[(size_t)hh * astr + t] = expf_exact(a.ex, tab_s, fsub(att[(size_t)hh * astr + t], mx[hh]));
    __syncthreads();
    // the denominators: the sequential sum over t = 0..pos, one lane per head
    if (lane == 0 && warp < KVM) s_inv[warp] = fdiv(1.0f, chain_sum_pipe(0.0f, att + (size_t)warp * astr, npos));
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < KVM; hh++)
        for (int t = tid; t < npos; t += ATTN_THREADS) att[(size_t)hh * astr + t] = fmul(att[(size_t)hh * astr + t], s_inv[hh]);

    // ---- out_i = sum_t w_t * v_t,i, sequential over t (ref src/model.c:252-256) ----
    const int ho = tid / hd, io = tid - ho * hd;
    const bool live = ho < KVM;
    const float *w = att + (size_t)(live ? ho : 0) * astr;
    float o = 0.0f;
    for (int c = 0; c < nch; c++) {
        const int c0 = c * AB_CH, n = min(AB_CH, npos - c0);
        if (c + 1 < nch) {
            ab_stage_v(buf0 + ((c + 1) & 1) * cbuf, vt, c0 + AB_CH, min(AB_CH, npos - c0 - AB_CH), hd);
            cp_async_wait_1();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();   // the chunk (and, for c = 0, the weights) are visible
        const T *vb = buf0 + (c & 1) * cbuf;
        if (live) {
            int t = 0;
            for (; t + 8 <= n; t += 8) {
                float ww[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) { ww[j] = w[c0 + t + j]; vv[j] = widen(vb[(size_t)(t + j) * hd + io]); }
#pragma unroll
                for (int j = 0; j < 8; j++) o = fadd(o, fmul(ww[j], vv[j]));
            }
            for (; t < n; t++) o = fadd(o, fmul(w[c0 + t], widen(vb[(size_t)t * hd + io])));
        }
        __syncthreads();   // the buffer is free for chunk c + 2
    }
    if (live) {
        const int gi = (kvh * KVM + ho) * hd + io;
        float dq;
        const int8_t q = quant_lane(o, &dq);   // hd % 32 == 0: a warp holds one block of one head
        a.bxq[(size_t)bt * a.k_pad + gi] = q;
        if (lane == 0) a.bxs[(size_t)(gi / 32) * a.n_pad + bt] = dq;
    }
}

}  // namespace emb
