// kernels.cuh — the token-step kernels (sm_100a).
//
// One decode step of a layer is five launches, each fused with the elementwise
// work around it so that no activation makes an extra HBM round trip:
//
//   gemv<IN_NORM, EPI_STORE>   RMSNorm(x)+Q8 quant -> [wq|wk|wv] -> q,k,v (+bias)
//   attn_decode                QK-norm, RoPE, KV store, scores, softmax, P.V,
//                              Q8 quant of the head outputs
//   gemv<IN_QUANT, EPI_RESID>  wo, x += .
//   gemv<IN_NORM, EPI_SWIGLU>  RMSNorm(x)+quant -> w1,w3 -> SiLU(g)*u -> Q8 quant
//   gemv<IN_QUANT, EPI_RESID>  w2, x += .
//
// and the step ends with gemv<IN_NORM, EPI_STORE> over lm_head (final norm
// fused) plus, for device-side greedy decoding, an argmax.
//
// Every fp32 result is bit-identical to emberllm's deterministic build: see the
// order notes at each step and the rules in common.cuh.
#pragma once

#include "common.cuh"

namespace emb {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_ROWS = 32;   // output rows per tile = one Q8 block of outputs
constexpr int ATTN_THREADS = 256;

enum { IN_RAW = 0, IN_NORM = 1, IN_QUANT = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };

// ctl words in device memory, read by the step's kernels (so one captured graph
// serves every position): [0] pos, [1] token, [2] number of greedy tokens
// written, [3] position of ids[0] during a prefill.
enum { CTL_POS = 0, CTL_TOK = 1, CTL_NOUT = 2, CTL_BASE = 3, CTL_WORDS = 4 };

// A weight matrix in the device layout: rows of quantized bytes (Q8_0: 32 int8
// per block; Q4_0: 16 bytes per block, nibble order as in the file) and, apart,
// the fp16 block scales [rows][cols/32]; or rows of fp32 values.
struct GemvSeg {
    const uint8_t *q;
    const __half *s;
    int dtype, rows;
    float *out;          // EPI_STORE / EPI_RESID destination, indexed by row
    const float *bias;   // EPI_STORE: optional, added after the dot (ref src/model.c:382-384)
};

struct GemvArgs {
    GemvSeg seg[3];
    int nseg, cols;
    int tiles[4];             // tiles[k] = first tile of segment k; tiles[nseg] = total
    int prefetch_tiles;       // tiles of its own each CTA prefetches into L2 before waiting
    // input
    const float *x;           // IN_RAW / IN_NORM: fp32 input
    const float *norm_w;      // IN_NORM
    float eps;
    const int8_t *xq;         // IN_QUANT: quantized input and its widened scales
    const float *xd;
    const float *xf;          // IN_QUANT: fp32 copy for fp32 weights (may be NULL)
    int8_t *xq_out;           // IN_RAW: CTA 0 also writes the quantized input (op tests)
    float *xd_out;
    // EPI_SWIGLU outputs: quantized h, its scales, fp32 h
    int8_t *hq;
    float *hd;
    float *hf;
    ExpfDev ex;
};

__host__ __device__ inline int gemv_p_stride(int nb) { return nb | 1; }

// dynamic shared memory of gemv_kernel
__host__ inline size_t gemv_smem_bytes(int cols, bool need_xf) {
    int nb = cols / 32;
    size_t b = ((size_t)cols + 15) / 16 * 16;                  // xq
    b += (size_t)(nb > 0 ? nb : 1) * 4;                         // xd
    b = (b + 15) / 16 * 16;
    if (need_xf) b += (size_t)cols * 4;                         // xf
    size_t p = (size_t)2 * GEMV_ROWS * gemv_p_stride(nb) * 4;   // P (also sq scratch)
    size_t sq = (size_t)cols * 4;
    b += p > sq ? p : sq;
    b += 2 * GEMV_ROWS * 4;                                     // row sums
    return b;
}

EMB_DEV GemvSeg pick_seg(const GemvArgs &a, int k) {
    return k == 0 ? a.seg[0] : (k == 1 ? a.seg[1] : a.seg[2]);
}

// int8 dot of one Q8_0 weight block (32 B) with one activation block
EMB_DEV int dot_q8_block(const uint8_t *w, const int8_t *xq) {
    uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(w));
    uint4 w1 = __ldg(reinterpret_cast<const uint4 *>(w) + 1);
    int4 a0 = reinterpret_cast<const int4 *>(xq)[0];
    int4 a1 = reinterpret_cast<const int4 *>(xq)[1];
    int acc = 0;
    acc = __dp4a((int)w0.x, a0.x, acc); acc = __dp4a((int)w0.y, a0.y, acc);
    acc = __dp4a((int)w0.z, a0.z, acc); acc = __dp4a((int)w0.w, a0.w, acc);
    acc = __dp4a((int)w1.x, a1.x, acc); acc = __dp4a((int)w1.y, a1.y, acc);
    acc = __dp4a((int)w1.z, a1.z, acc); acc = __dp4a((int)w1.w, a1.w, acc);
    return acc;
}

// Q4_0 block (16 B): element i is nibble (byte i & 15) - 8, element i+16 is
// (byte i >> 4) - 8 (ref src/kernels.c:175-179). Unsigned nibbles fit in a
// signed byte, so sum((n-8)*a) = sum(n*a) - 8*sum(a), all exact in int32.
EMB_DEV int dot_q4_block(const uint8_t *w, const int8_t *xq) {
    uint4 v = __ldg(reinterpret_cast<const uint4 *>(w));
    int4 a0 = reinterpret_cast<const int4 *>(xq)[0];
    int4 a1 = reinterpret_cast<const int4 *>(xq)[1];
    const uint32_t m = 0x0F0F0F0Fu;
    int acc = 0;
    acc = __dp4a((int)(v.x & m), a0.x, acc); acc = __dp4a((int)(v.y & m), a0.y, acc);
    acc = __dp4a((int)(v.z & m), a0.z, acc); acc = __dp4a((int)(v.w & m), a0.w, acc);
    acc = __dp4a((int)((v.x >> 4) & m), a1.x, acc); acc = __dp4a((int)((v.y >> 4) & m), a1.y, acc);
    acc = __dp4a((int)((v.z >> 4) & m), a1.z, acc); acc = __dp4a((int)((v.w >> 4) & m), a1.w, acc);
    int sa = 0;
    const int ones = 0x01010101;
    sa = __dp4a(a0.x, ones, sa); sa = __dp4a(a0.y, ones, sa); sa = __dp4a(a0.z, ones, sa);
    sa = __dp4a(a0.w, ones, sa); sa = __dp4a(a1.x, ones, sa); sa = __dp4a(a1.y, ones, sa);
    sa = __dp4a(a1.z, ones, sa); sa = __dp4a(a1.w, ones, sa);
    return acc - 8 * sa;
}

// Issue L2 prefetches for one tile of a segment (weights are read-only, so this
// is safe before the dependency wait).
EMB_DEV void prefetch_tile(const GemvSeg &g, int row0, int cols) {
    int nrows = min(GEMV_ROWS, g.rows - row0);
    if (nrows <= 0 || g.dtype == EMBER_DT_F32) return;
    size_t rb = qrow_bytes(g.dtype, cols);
    uint32_t qbytes = (uint32_t)(rb * (size_t)nrows) & ~15u;
    if (qbytes) prefetch_l2(g.q + rb * (size_t)row0, qbytes);
    int nb = cols / 32;
    uint32_t sbytes = (uint32_t)((size_t)nrows * nb * 2) & ~15u;
    if (sbytes) prefetch_l2(g.s + (size_t)row0 * nb, sbytes);
}

template <int IN, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int cols = a.cols, nb = cols / 32, pstride = gemv_p_stride(nb);
    const int total = a.tiles[a.nseg];
    const int ntiles_seg = EPI == EPI_SWIGLU ? total : 0;  // swiglu: tile t covers seg0 and seg1

    bool has_f32 = false;
    for (int k = 0; k < (EPI == EPI_SWIGLU ? 2 : a.nseg); k++) has_f32 |= pick_seg(a, k).dtype == EMBER_DT_F32;
    const bool need_xf = IN != IN_QUANT || has_f32;

    int8_t *xq_s = reinterpret_cast<int8_t *>(smem);
    size_t off = ((size_t)cols + 15) / 16 * 16;
    float *xd_s = reinterpret_cast<float *>(smem + off);
    off = (off + (size_t)(nb > 0 ? nb : 1) * 4 + 15) / 16 * 16;
    float *xf_s = reinterpret_cast<float *>(smem + off);
    if (need_xf) off += (size_t)cols * 4;
    float *P = reinterpret_cast<float *>(smem + off);
    size_t psz = (size_t)2 * GEMV_ROWS * pstride * 4, sqsz = (size_t)cols * 4;
    off += psz > sqsz ? psz : sqsz;
    float *rowsum = reinterpret_cast<float *>(smem + off);
    __shared__ float s_scale;

    pdl_launch_dependents();
    if (tid == 0) {
        int k = 0;
        for (int t = blockIdx.x, n = 0; t < total && n < a.prefetch_tiles; t += gridDim.x, n++) {
            if (EPI == EPI_SWIGLU) {
                prefetch_tile(a.seg[0], t * GEMV_ROWS, cols);
                prefetch_tile(a.seg[1], t * GEMV_ROWS, cols);
            } else {
                while (k + 1 < a.nseg && t >= a.tiles[k + 1]) k++;
                prefetch_tile(pick_seg(a, k), (t - a.tiles[k]) * GEMV_ROWS, cols);
            }
        }
    }
    pdl_wait();

    // ---- prologue: the Q8_0 activation (and fp32 copy) in shared memory ----
    if (IN == IN_QUANT) {
        for (int i = tid; i < cols / 16; i += GEMV_THREADS)
            reinterpret_cast<int4 *>(xq_s)[i] = reinterpret_cast<const int4 *>(a.xq)[i];
        for (int i = tid; i < nb; i += GEMV_THREADS) xd_s[i] = a.xd[i];
        if (need_xf)
            for (int i = tid; i < cols; i += GEMV_THREADS) xf_s[i] = a.xf[i];
    } else {
        for (int i = tid; i < cols; i += GEMV_THREADS) xf_s[i] = a.x[i];
        if (IN == IN_NORM) {
            // RMSNorm (ref src/model.c:50-55): products in parallel, then the sum of
            // squares as ONE sequential chain in index order, as the reference adds.
            float *sq = P;
            __syncthreads();
            for (int i = tid; i < cols; i += GEMV_THREADS) sq[i] = fmul(xf_s[i], xf_s[i]);
            __syncthreads();
            if (tid == 0) {
                float ss = 0.0f;
#pragma unroll 16
                for (int i = 0; i < cols; i++) ss = fadd(ss, sq[i]);
                s_scale = rms_scale(ss, cols, a.eps);
            }
            __syncthreads();
            const float sc = s_scale;
            for (int i = tid; i < cols; i += GEMV_THREADS)
                xf_s[i] = fmul(fmul(xf_s[i], sc), a.norm_w[i]);   // (x*scale)*w
        }
        __syncthreads();
        // quantize the activation, one warp per 32-block (ref src/kernels.c:211)
        const int warp = tid >> 5, lane = tid & 31;
        for (int b = warp; b < nb; b += GEMV_THREADS / 32) {
            float dq;
            int8_t q = quant_lane(xf_s[b * 32 + lane], &dq);
            xq_s[b * 32 + lane] = q;
            if (lane == 0) xd_s[b] = dq;
            if (IN == IN_RAW && blockIdx.x == 0 && a.xq_out) {
                a.xq_out[b * 32 + lane] = q;
                if (lane == 0) a.xd_out[b] = dq;
            }
        }
    }
    __syncthreads();

    // ---- tiles ----
    int k = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
        int nsub, row0;
        GemvSeg g0, g1;
        if (EPI == EPI_SWIGLU) {
            g0 = a.seg[0];
            g1 = a.seg[1];
            row0 = t * GEMV_ROWS;
            nsub = 2;
        } else {
            while (k + 1 < a.nseg && t >= a.tiles[k + 1]) k++;
            g0 = pick_seg(a, k);
            g1 = g0;
            row0 = (t - a.tiles[k]) * GEMV_ROWS;
            nsub = 1;
        }
        (void)ntiles_seg;
        const int nrows = min(GEMV_ROWS, g0.rows - row0);
        const int rows_total = nsub * GEMV_ROWS;

        // phase 1: per (row, block) products ((float)acc * d_w) * d_x into P
        for (int sub = 0; sub < nsub; sub++) {
            const GemvSeg &g = sub == 0 ? g0 : g1;
            if (g.dtype == EMBER_DT_F32) {
                // fp32 weights: the reference's scalar dot, one chain per row over
                // all inputs in order (ref src/kernels.c:143-146)
                if (tid < nrows) {
                    const float *w = reinterpret_cast<const float *>(g.q) + (size_t)(row0 + tid) * cols;
                    float s = 0.0f;
                    for (int i = 0; i < cols; i++) s = fadd(s, fmul(__ldg(w + i), xf_s[i]));
                    rowsum[sub * GEMV_ROWS + tid] = s;
                }
                continue;
            }
            const size_t rb = qrow_bytes(g.dtype, cols);
            const uint8_t *tq = g.q + rb * (size_t)row0;
            const __half *ts = g.s + (size_t)row0 * nb;
            const int items = nrows * nb;
            const int bbytes = g.dtype == EMBER_DT_Q8_0 ? 32 : 16;
            float *Ps = P + (size_t)sub * GEMV_ROWS * pstride;
            for (int j = tid; j < items; j += GEMV_THREADS) {
                const int r = j / nb, b = j - r * nb;
                const uint8_t *wb = tq + (size_t)r * rb + (size_t)b * bbytes;
                int acc = g.dtype == EMBER_DT_Q8_0 ? dot_q8_block(wb, xq_s + b * 32)
                                                   : dot_q4_block(wb, xq_s + b * 32);
                float dw = __half2float(ts[j]);
                Ps[r * pstride + b] = fmul(fmul(__int2float_rn(acc), dw), xd_s[b]);
            }
        }
        __syncthreads();
        // phase 2: each row's block terms summed in block order (ref src/kernels.c:152-164)
        if (tid < rows_total) {
            const int sub = tid / GEMV_ROWS, r = tid - sub * GEMV_ROWS;
            const GemvSeg &g = sub == 0 ? g0 : g1;
            if (r < nrows && g.dtype != EMBER_DT_F32) {
                const float *pr = P + ((size_t)sub * GEMV_ROWS + r) * pstride;
                float s = 0.0f;
#pragma unroll 8
                for (int b = 0; b < nb; b++) s = fadd(s, pr[b]);
                rowsum[tid] = s;
            }
        }
        __syncthreads();
        // epilogue
        if (EPI == EPI_SWIGLU) {
            if (tid < 32) {
                // h = SiLU(g) * u = g / (1 + expf(-g)) * u (ref src/model.c:403-406)
                float h = 0.0f;
                if (tid < nrows) {
                    float gv = rowsum[tid], uv = rowsum[GEMV_ROWS + tid];
                    float e = expf_exact(a.ex, -gv);
                    h = fmul(fdiv(gv, fadd(1.0f, e)), uv);
                    if (a.hf) a.hf[row0 + tid] = h;
                }
                // the next matmul's Q8 quantization of this 32-block of h
                float dq;
                int8_t q = quant_lane(h, &dq);
                if (tid < nrows) a.hq[row0 + tid] = q;
                if (tid == 0) a.hd[row0 / 32] = dq;
            }
        } else if (tid < nrows) {
            float s = rowsum[tid];
            if (EPI == EPI_RESID) {
                g0.out[row0 + tid] = fadd(g0.out[row0 + tid], s);    // x += y (ref :398, :408)
            } else {
                if (g0.bias) s = fadd(s, g0.bias[row0 + tid]);
                g0.out[row0 + tid] = s;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- attention ----

struct AttnArgs {
    const float *q, *k, *v;        // this position's projections (bias already added)
    void *kc, *vc;                 // this layer's cache: [n_kv][ctx][hd], fp32 or fp16
    const float *q_norm, *k_norm;  // QK-norm weights [hd] or NULL
    const float2 *rope;            // [ctx][hd/2] (cos, sin)
    const int *ctl;
    float *att;                    // scratch [n_heads][ctx]
    int8_t *oq;                    // outputs: Q8 of the head outputs [n_heads*hd] ...
    float *od;                     //   ... their scales [n_heads*hd/32]
    float *of;                     //   ... and the fp32 values
    int nh, nkv, hd, ctx, neox;
    float eps;
    ExpfDev ex;
};

EMB_DEV float kv_load(const float *p) { return *p; }
EMB_DEV float kv_load(const __half *p) { return __half2float(*p); }

EMB_DEV void kv_load4(const float *p, float *o) {
    float4 v = *reinterpret_cast<const float4 *>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
EMB_DEV void kv_load4(const __half *p, float *o) {
    uint2 u = *reinterpret_cast<const uint2 *>(p);
    __half2 a = *reinterpret_cast<__half2 *>(&u.x), b = *reinterpret_cast<__half2 *>(&u.y);
    float2 fa = __half22float2(a), fb = __half22float2(b);
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
}

// the value stored in the cache: fp32 as is, or fp16 rounded to nearest even
// (ref src/model.c:43, ember_f16c)
EMB_DEV void kv_round(float v, float *out) { *out = v; }
EMB_DEV void kv_round(float v, __half *out) { *out = __float2half_rn(v); }
EMB_DEV float kv_widen(float v) { return v; }
EMB_DEV float kv_widen(__half v) { return __half2float(v); }

// One query position over the cache for one head (ref src/model.c:221-259).
template <typename T>
__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const AttnArgs a) {
    __shared__ float qs[256], ks[256], vs[256];
    __shared__ float red[ATTN_THREADS / 32];
    __shared__ float s_q, s_k, s_max, s_inv;
    const int h = blockIdx.x, tid = threadIdx.x, hd = a.hd;
    const int kvh = h / (a.nh / a.nkv);
    pdl_launch_dependents();
    pdl_wait();
    const int pos = a.ctl[CTL_POS];
    T *kc = reinterpret_cast<T *>(a.kc) + (size_t)kvh * a.ctx * hd;
    T *vc = reinterpret_cast<T *>(a.vc) + (size_t)kvh * a.ctx * hd;

    if (tid < hd) {
        qs[tid] = a.q[h * hd + tid];
        ks[tid] = a.k[kvh * hd + tid];
        vs[tid] = a.v[kvh * hd + tid];
    }
    __syncthreads();
    if (a.q_norm) {
        // per-head RMSNorm of q and k, in place (ref src/model.c:386-389); the two
        // sequential sums run on different warps
        if (tid == 0) {
            float ss = 0.0f;
            for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(qs[i], qs[i]));
            s_q = rms_scale(ss, hd, a.eps);
        } else if (tid == 32) {
            float ss = 0.0f;
            for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(ks[i], ks[i]));
            s_k = rms_scale(ss, hd, a.eps);
        }
        __syncthreads();
        if (tid < hd) {
            qs[tid] = fmul(fmul(qs[tid], s_q), a.q_norm[tid]);
            ks[tid] = fmul(fmul(ks[tid], s_k), a.k_norm[tid]);
        }
        __syncthreads();
    }
    // RoPE (ref src/model.c:66-80) with the host-built cos/sin table
    if (tid < hd / 2) {
        const int ia = a.neox ? tid : 2 * tid, ib = a.neox ? tid + hd / 2 : 2 * tid + 1;
        const float2 cs = a.rope[(size_t)pos * (hd / 2) + tid];
        float v0 = qs[ia], v1 = qs[ib];
        qs[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        qs[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
        v0 = ks[ia]; v1 = ks[ib];
        ks[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        ks[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
    }
    __syncthreads();
    // KV store (ref src/model.c:39-48): the cache holds fp32 or RNE fp16; attention
    // reads the stored values, including at t == pos
    if (tid < hd) {
        T kt, vt;
        kv_round(ks[tid], &kt);
        kv_round(vs[tid], &vt);
        ks[tid] = kv_widen(kt);
        vs[tid] = kv_widen(vt);
        if (h % (a.nh / a.nkv) == 0) {
            kc[(size_t)pos * hd + tid] = kt;
            vc[(size_t)pos * hd + tid] = vt;
        }
    }
    __syncthreads();

    // scores: sc = sum_i q_i*k_i in index order, then * (1/sqrt(hd))
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    float *att = a.att + (size_t)h * a.ctx;
    float tmax = -INFINITY;
    for (int t = tid; t <= pos; t += ATTN_THREADS) {
        float sc = 0.0f;
        if (t == pos) {
            for (int i = 0; i < hd; i++) sc = fadd(sc, fmul(qs[i], ks[i]));
        } else {
            const T *kr = kc + (size_t)t * hd;
            for (int i = 0; i < hd; i += 4) {
                float kk[4];
                kv_load4(kr + i, kk);
                sc = fadd(sc, fmul(qs[i], kk[0]));
                sc = fadd(sc, fmul(qs[i + 1], kk[1]));
                sc = fadd(sc, fmul(qs[i + 2], kk[2]));
                sc = fadd(sc, fmul(qs[i + 3], kk[3]));
            }
        }
        sc = fmul(sc, inv_sqrt);
        att[t] = sc;
        tmax = fmaxf(tmax, sc);
    }
    // softmax (ref src/model.c:57-64): max is order-free
    tmax = warp_max(tmax);
    if ((tid & 31) == 0) red[tid >> 5] = tmax;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < ATTN_THREADS / 32; w++) m = fmaxf(m, red[w]);
        s_max = m;
    }
    __syncthreads();
    const float mx = s_max;
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = expf_exact(a.ex, fsub(att[t], mx));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;                            // sequential, t = 0..pos
#pragma unroll 8
        for (int t = 0; t <= pos; t++) sum = fadd(sum, att[t]);
        s_inv = fdiv(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = fmul(att[t], inv);
    __syncthreads();

    // out_i = sum_t w_t * v_t,i, sequential over t (ref src/model.c:252-256)
    if (tid < hd) {
        float o = 0.0f;
        const T *vcol = vc + tid;
#pragma unroll 8
        for (int t = 0; t < pos; t++) o = fadd(o, fmul(att[t], kv_load(vcol + (size_t)t * hd)));
        o = fadd(o, fmul(att[pos], vs[tid]));
        const int gi = h * hd + tid;
        if (a.of) a.of[gi] = o;
        float dq;
        int8_t q = quant_lane(o, &dq);   // hd % 32 == 0: each warp owns one block
        a.oq[gi] = q;
        if ((tid & 31) == 0) a.od[gi / 32] = dq;
    }
}

// ---------------------------------------------------------------- embedding ----

struct EmbedArgs {
    const uint8_t *q;     // Q8_0 rows (int8) or fp32 rows
    const __half *s;
    int dtype, dim;
    int *ctl;
    const int *ids;       // prefill: token = ids[pos - ctl[CTL_BASE]]
    float *x;
};

// x = the token's embedding row, dequantized as q*d (ref src/model.c:83-100)
__global__ void __launch_bounds__(256) embed_kernel(const EmbedArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int pos = a.ctl[CTL_POS];
    const int tok = a.ids ? a.ids[pos - a.ctl[CTL_BASE]] : a.ctl[CTL_TOK];
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
        if (a.dtype == EMBER_DT_F32) {
            a.x[i] = reinterpret_cast<const float *>(a.q)[(size_t)tok * a.dim + i];
        } else {
            int8_t q = reinterpret_cast<const int8_t *>(a.q)[(size_t)tok * a.dim + i];
            float d = __half2float(a.s[(size_t)tok * (a.dim / 32) + i / 32]);
            a.x[i] = fmul((float)q, d);
        }
    }
}

// ---------------------------------------------------------------- argmax -------

struct ArgmaxArgs {
    const float *logits;
    int n;
    float *part_v;        // [gridDim.x]
    int *part_i;
    unsigned *ticket;     // zero between launches
    int *ctl;             // advance: ctl[TOK] = argmax, ctl[POS] += 1, out[ctl[NOUT]++] = argmax
    int *out;
};

// first index of the strict maximum (ref src/sample.c:114-118)
EMB_DEV void am_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__global__ void __launch_bounds__(256) argmax_advance_kernel(const ArgmaxArgs a) {
    __shared__ float sv[256];
    __shared__ int si[256];
    __shared__ bool last;
    pdl_launch_dependents();
    pdl_wait();
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x)
        am_merge(bv, bi, a.logits[i], i);
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            float v = sv[threadIdx.x + st];
            int i = si[threadIdx.x + st];
            float cv = sv[threadIdx.x];
            int ci = si[threadIdx.x];
            am_merge(cv, ci, v, i);
            sv[threadIdx.x] = cv;
            si[threadIdx.x] = ci;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        a.part_v[blockIdx.x] = sv[0];
        a.part_i[blockIdx.x] = si[0];
        __threadfence();
        unsigned t = atomicAdd(a.ticket, 1u);
        last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float v = -INFINITY;
        int idx = 0x7FFFFFFF;
        for (int b = 0; b < (int)gridDim.x; b++) {
            float pv = *(volatile float *)&a.part_v[b];
            int pi = *(volatile int *)&a.part_i[b];
            am_merge(v, idx, pv, pi);
        }
        if (idx == 0x7FFFFFFF) idx = 0;   // all -inf/NaN: the reference keeps index 0
        a.ctl[CTL_TOK] = idx;
        a.ctl[CTL_POS] += 1;
        if (a.out) a.out[a.ctl[CTL_NOUT]] = idx;
        a.ctl[CTL_NOUT] += 1;
        *a.ticket = 0;
    }
}

// prefill bookkeeping between steps: advance the position
__global__ void advance_kernel(int *ctl) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) ctl[CTL_POS] += 1;
}

}  // namespace emb
