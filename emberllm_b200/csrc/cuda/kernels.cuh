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
// Data movement. Weight tiles (R consecutive rows: their quant bytes and their
// fp16 scales, each a contiguous range in the device layout) are moved into
// shared memory by bulk asynchronous copies (TMA, cp.async.bulk) that complete
// on an mbarrier. The copies of a CTA's first tiles are issued BEFORE the
// programmatic-launch wait, so they overlap the previous kernel; later tiles
// stream through a ring of stages. Attention stages each chunk of the cache the
// same way. Every wait on an mbarrier is bounded (common.cuh).
//
// Every fp32 result is bit-identical to emberllm's deterministic build: see the
// order notes at each step and the rules in common.cuh.
#pragma once

#include "common.cuh"

namespace emb {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_MAX_ROWS = 32;     // rows per tile (SwiGLU: exactly one Q8 block of h)
constexpr int GEMV_MAX_STAGES = 4;
constexpr int ATTN_THREADS = 256;

enum { IN_RAW = 0, IN_NORM = 1, IN_QUANT = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };


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
    int rows;                 // rows per tile R (<= 32; SwiGLU: 32)
    int tiles[4];             // tiles[k] = first tile of segment k; tiles[nseg] = total
    int stages;               // shared-memory ring depth (quantized weights)
    int stage_bytes;          // bytes of one stage (all sub-tiles)
    int quantized;            // 1: Q8_0/Q4_0 segments (bulk copies); 0: fp32 segments
    // input
    const float *x;           // IN_RAW / IN_NORM: fp32 input
    const float *norm_w;      // IN_NORM
    float eps;
    const int8_t *xq;         // IN_QUANT: quantized input and its widened scales
    const float *xd;
    const float *xf;          // IN_QUANT: fp32 copy for fp32 weights (may be NULL)
    int8_t *xq_out;           // IN_RAW: CTA 0 also writes the quantized input (op tests)
    float *xd_out;
    // EPI_SWIGLU outputs: quantized h, its scales, fp32 h (fp32 only when needed)
    int8_t *hq;
    float *hd;
    float *hf;
    int *err;
    ExpfDev ex;
};

__host__ __device__ inline int gemv_p_stride(int nb) { return nb | 1; }
__host__ __device__ inline size_t pad16(size_t n) { return (n + 15) / 16 * 16; }

// bytes of one sub-tile (R rows of one matrix) inside a stage
__host__ __device__ inline size_t gemv_sub_bytes(int dtype, int rows, int cols) {
    return pad16((size_t)rows * qrow_bytes(dtype, cols)) + pad16((size_t)rows * (cols / 32) * 2);
}

// bytes of the region that holds the tile products P, and during an RMSNorm
// prologue (before any tile) the norm weights and the squares instead
__host__ __device__ inline size_t gemv_p_bytes(int cols, bool in_norm) {
    size_t p = (size_t)2 * GEMV_MAX_ROWS * gemv_p_stride(cols / 32) * 4;
    // the prologue's norm weights and squares (in_norm)
    size_t pro = in_norm ? (size_t)cols * 8 : 0;
    return pad16(p > pro ? p : pro);
}

// dynamic shared memory of ember_q8_gemv_kernel
__host__ inline size_t gemv_smem_bytes(const GemvArgs &a, bool need_xf, bool in_norm) {
    const int cols = a.cols, nb = cols / 32;
    size_t b = a.quantized ? (size_t)a.stages * a.stage_bytes : 0;
    b += pad16(cols);                                           // xq
    b += pad16((size_t)(nb > 0 ? nb : 1) * 4);                  // xd
    if (need_xf) b += (size_t)cols * 4;                         // xf
    b += gemv_p_bytes(cols, in_norm);                           // P / prologue scratch
    b += 2 * GEMV_MAX_ROWS * 4;                                 // row sums
    return b;
}

EMB_DEV GemvSeg pick_seg(const GemvArgs &a, int k) {
    return k == 0 ? a.seg[0] : (k == 1 ? a.seg[1] : a.seg[2]);
}

// Which segment / first row / row count a tile covers, for sub-tile `sub`.
struct TileRef {
    GemvSeg g;
    int row0, nrows;
};

template <int EPI>
EMB_DEV TileRef tile_ref(const GemvArgs &a, int t, int sub) {
    TileRef r;
    int k = 0;
    if (EPI == EPI_SWIGLU) {
        k = sub;
        r.row0 = t * a.rows;
    } else {
        while (k + 1 < a.nseg && t >= a.tiles[k + 1]) k++;
        r.row0 = (t - a.tiles[k]) * a.rows;
    }
    r.g = pick_seg(a, k);
    r.nrows = min(a.rows, r.g.rows - r.row0);
    return r;
}

// Thread 0: bulk-copy tile t (all its sub-tiles) into stage buffer `dst`.
template <int EPI>
EMB_DEV void issue_tile(const GemvArgs &a, int t, unsigned char *dst, uint64_t *bar) {
    constexpr int nsub = EPI == EPI_SWIGLU ? 2 : 1;
    const int nb = a.cols / 32;
    uint32_t total = 0;
    TileRef tr[nsub];
#pragma unroll
    for (int sub = 0; sub < nsub; sub++) {
        tr[sub] = tile_ref<EPI>(a, t, sub);
        total += (uint32_t)(tr[sub].nrows * qrow_bytes(tr[sub].g.dtype, a.cols));
        total += (uint32_t)pad16((size_t)tr[sub].nrows * nb * 2);
    }
    mbar_expect_tx(bar, total);
    size_t off = 0;
#pragma unroll
    for (int sub = 0; sub < nsub; sub++) {
        const GemvSeg &g = tr[sub].g;
        const size_t rb = qrow_bytes(g.dtype, a.cols);
        const uint32_t qb = (uint32_t)(tr[sub].nrows * rb);
        const uint32_t sb = (uint32_t)pad16((size_t)tr[sub].nrows * nb * 2);
        bulk_g2s(dst + off, g.q + rb * (size_t)tr[sub].row0, qb, bar);
        // scale rows are padded on the device by 16 bytes, so rounding up is in bounds
        bulk_g2s(dst + off + pad16((size_t)a.rows * rb), g.s + (size_t)tr[sub].row0 * nb, sb, bar);
        off += gemv_sub_bytes(g.dtype, a.rows, a.cols);
    }
}

template <int IN, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) ember_q8_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[GEMV_MAX_STAGES];
    __shared__ double tab_s[EPI == EPI_SWIGLU ? 64 : 1];
    constexpr int nsub = EPI == EPI_SWIGLU ? 2 : 1;
    const int tid = threadIdx.x, R = a.rows;
    const int cols = a.cols, nb = cols / 32, pstride = gemv_p_stride(nb);
    const int total = a.tiles[a.nseg];
    const int my_tiles = (int)blockIdx.x < total ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const bool need_xf = IN != IN_QUANT || !a.quantized;
    const int S = a.quantized ? a.stages : 0;

    unsigned char *stage0 = smem;
    size_t off = (size_t)S * a.stage_bytes;
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + off);
    off += pad16(cols);
    float *xd_s = reinterpret_cast<float *>(smem + off);
    off += pad16((size_t)(nb > 0 ? nb : 1) * 4);
    float *xf_s = reinterpret_cast<float *>(smem + off);
    if (need_xf) off += (size_t)cols * 4;
    float *P = reinterpret_cast<float *>(smem + off);
    off += gemv_p_bytes(cols, IN == IN_NORM);
    float *rowsum = reinterpret_cast<float *>(smem + off);

    // probe kind: 0 q/k/v, 5 lm_head, 1 w1/w3, 2 wo/w2, 3 op-level
    const int PK = IN == IN_NORM ? (EPI == EPI_SWIGLU ? 1 : (a.nseg == 1 ? 5 : 0)) : (IN == IN_QUANT ? 2 : 3);
    EMB_PROBE(PK, 0);
    (void)PK;
    // ---- pre-wait: only weights (the tiles and the norm vector) ----
    if (S > 0 && tid == 0) {
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int k = 0; k < S && k < my_tiles; k++)
            issue_tile<EPI>(a, blockIdx.x + k * gridDim.x, stage0 + (size_t)k * a.stage_bytes, &bars[k]);
    }
    // until the tiles need P: the norm weights
    float *nw_s = P;
    if (IN == IN_NORM)
        for (int i = tid; i < cols; i += GEMV_THREADS) nw_s[i] = a.norm_w[i];
    if (EPI == EPI_SWIGLU) expf_table_load(tab_s, a.ex);
    // residual rows of the first tile: x was last written two or more launches
    // back (w2 of the previous layer before wo; wo before w13, w2), so it may be
    // read before the wait
    float resid0 = 0.0f;
    if (EPI == EPI_RESID && my_tiles > 0 && tid < R) {
        const TileRef t0 = tile_ref<EPI>(a, blockIdx.x, 0);
        if (tid < t0.nrows) resid0 = t0.g.out[t0.row0 + tid];
    }
    EMB_PROBE(PK, 1);
    pdl_wait_then_release();
    EMB_PROBE(PK, 2);

    // ---- prologue: the Q8_0 activation (and fp32 copy) in shared memory ----
    if (IN == IN_QUANT) {
        for (int i = tid; i < cols / 16; i += GEMV_THREADS)
            reinterpret_cast<int4 *>(xq_s)[i] = reinterpret_cast<const int4 *>(a.xq)[i];
        for (int i = tid; i < nb; i += GEMV_THREADS) xd_s[i] = a.xd[i];
        if (need_xf)
            for (int i = tid; i < cols; i += GEMV_THREADS) xf_s[i] = a.xf[i];
    } else {
        // RMSNorm (ref src/model.c:50-55): the sum of squares in index order, as
        // the reference adds, by split_chain_sum over the squares (after the norm
        // weights in the prologue scratch)
        float *sq_s = nw_s + cols;
        if (IN == IN_NORM) {
            for (int i = tid; i < cols; i += GEMV_THREADS) {
                const float v = a.x[i];
                xf_s[i] = v;
                sq_s[i] = fmul(v, v);
            }
        } else {
            for (int i = tid; i < cols; i += GEMV_THREADS) xf_s[i] = a.x[i];
        }
        if (IN == IN_NORM) {
            __syncthreads();
            EMB_PROBE(PK, 3);
            const float sc = rms_scale(split_chain_sum<GEMV_THREADS>(sq_s, cols), cols, a.eps);
            EMB_PROBE(PK, 4);
            for (int i = tid; i < cols; i += GEMV_THREADS)
                xf_s[i] = fmul(fmul(xf_s[i], sc), nw_s[i]);   // (x*scale)*w
        }
        __syncthreads();
        // quantize the activation (ref src/kernels.c:211): eight threads per
        // 32-block, four elements each, every block at once
        for (int base = 0; base < nb * 8; base += GEMV_THREADS) {
            const int q8 = base + tid;
            const bool act = q8 < nb * 8;
            const unsigned mask = __ballot_sync(0xffffffffu, act);
            if (act) {
                const int b = q8 >> 3, sub = q8 & 7;
                float dq;
                const uint32_t packed = quant_quad(reinterpret_cast<const float4 *>(xf_s + b * 32)[sub], mask, &dq);
                reinterpret_cast<uint32_t *>(xq_s + b * 32)[sub] = packed;
                if (sub == 0) xd_s[b] = dq;
                if (IN == IN_RAW && blockIdx.x == 0 && a.xq_out) {
                    reinterpret_cast<uint32_t *>(a.xq_out + b * 32)[sub] = packed;
                    if (sub == 0) a.xd_out[b] = dq;
                }
            }
        }
    }
    __syncthreads();
    EMB_PROBE(PK, 5);

    // ---- tiles ----
    for (int k = 0; k < my_tiles; k++) {
        const int t = blockIdx.x + k * gridDim.x;
        TileRef tr[nsub];
#pragma unroll
        for (int sub = 0; sub < nsub; sub++) tr[sub] = tile_ref<EPI>(a, t, sub);
        const int nrows = tr[0].nrows;

        if (S > 0) {
            const int st = k % S;
            const unsigned char *stage = stage0 + (size_t)st * a.stage_bytes;
            mbar_wait_cta(&bars[st], (uint32_t)((k / S) & 1), a.err, ERR_GEMV_WAIT);
            if (k == 0) EMB_PROBE(PK, 6);
            // phase 1: per (row, block) terms ((float)acc * d_w) * d_x into P
            size_t soff = 0;
#pragma unroll
            for (int sub = 0; sub < nsub; sub++) {
                const GemvSeg &g = tr[sub].g;
                const size_t rb = qrow_bytes(g.dtype, cols);
                const uint8_t *tq = stage + soff;
                const __half *ts = reinterpret_cast<const __half *>(stage + soff + pad16((size_t)R * rb));
                const int items = tr[sub].nrows * nb;
                float *Ps = P + (size_t)sub * GEMV_MAX_ROWS * pstride;
                if (g.dtype == EMBER_DT_Q8_0) {
                    for (int j = tid; j < items; j += GEMV_THREADS) {
                        const int r = j / nb, b = j - r * nb;
                        int acc = dot_q8_block(tq + (size_t)r * rb + (size_t)b * 32, xq_s + b * 32);
                        Ps[r * pstride + b] = fmul(fmul(__int2float_rn(acc), __half2float(ts[j])), xd_s[b]);
                    }
                } else {
                    for (int j = tid; j < items; j += GEMV_THREADS) {
                        const int r = j / nb, b = j - r * nb;
                        int acc = dot_q4_block(tq + (size_t)r * rb + (size_t)b * 16, xq_s + b * 32);
                        Ps[r * pstride + b] = fmul(fmul(__int2float_rn(acc), __half2float(ts[j])), xd_s[b]);
                    }
                }
                soff += gemv_sub_bytes(g.dtype, R, cols);
            }
            __syncthreads();
            if (k == 0) EMB_PROBE(PK, 7);
            // the stage is free: refill it with this CTA's tile k + S
            if (tid == 0 && k + S < my_tiles) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_tile<EPI>(a, blockIdx.x + (k + S) * gridDim.x, stage0 + (size_t)st * a.stage_bytes, &bars[st]);
            }
            // phase 2: each row's block terms summed in block order (ref src/kernels.c:152-164)
            if (tid < nsub * R) {
                const int sub = tid / R, r = tid - sub * R;
                if (r < tr[sub].nrows) {
                    const float *pr = P + ((size_t)sub * GEMV_MAX_ROWS + r) * pstride;
                    rowsum[sub * GEMV_MAX_ROWS + r] = chain_sum_pipe(0.0f, pr, nb);
                }
            }
        } else {
            // fp32 weights: the reference's scalar dot, one chain per row over
            // all inputs in order (ref src/kernels.c:143-146)
            if (tid < nsub * R) {
                const int sub = tid / R, r = tid - sub * R;
                if (r < tr[sub].nrows) {
                    const float *w = reinterpret_cast<const float *>(tr[sub].g.q) + (size_t)(tr[sub].row0 + r) * cols;
                    float s = 0.0f;
                    for (int i = 0; i < cols; i++) s = fadd(s, fmul(__ldg(w + i), xf_s[i]));
                    rowsum[sub * GEMV_MAX_ROWS + r] = s;
                }
            }
        }
        __syncthreads();
        if (k == 0) EMB_PROBE(PK, 8);
        // epilogue
        const int row0 = tr[0].row0;
        if (EPI == EPI_SWIGLU) {
            if (tid < 32) {
                // h = SiLU(g) * u = g / (1 + expf(-g)) * u (ref src/model.c:403-406)
                float h = 0.0f;
                if (tid < nrows) {
                    float gv = rowsum[tid], uv = rowsum[GEMV_MAX_ROWS + tid];
                    float e = expf_exact(a.ex, tab_s, -gv);
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
            const GemvSeg &g = tr[0].g;
            if (EPI == EPI_RESID) {
                const float x = k == 0 ? resid0 : g.out[row0 + tid];
                g.out[row0 + tid] = fadd(x, s);    // x += y (ref :398, :408)
            } else {
                if (g.bias) s = fadd(s, g.bias[row0 + tid]);
                g.out[row0 + tid] = s;
            }
        }
        __syncthreads();
        if (k == 0) EMB_PROBE(PK, 9);
    }
    EMB_PROBE(PK, 10);
}

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
template <typename T>
__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float qs[256], ks[256], vs[256], qn_s[256], kn_s[256];
    __shared__ float2 cs_s[128];
    __shared__ float red[ATTN_THREADS / 32];
    __shared__ float s_q, s_k, s_max, s_inv;
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
    const int pos = a.ctl[CTL_POS];   // written by the host or the previous step's tail
    T *kt = reinterpret_cast<T *>(a.kc) + (size_t)kvh * hd * a.kstride;
    T *vt = reinterpret_cast<T *>(a.vc) + (size_t)kvh * a.ctx * hd;
    if (tid < hd) {
        qn_s[tid] = a.q_norm ? a.q_norm[tid] : 0.0f;
        kn_s[tid] = a.k_norm ? a.k_norm[tid] : 0.0f;
    }
    if (tid < hd / 2) cs_s[tid] = a.rope[(size_t)pos * (hd / 2) + tid];
    expf_table_load(tab_s, a.ex);
    __syncthreads();
    const int nchunks = (pos + CH - 1) / CH;
    const int n0 = min(CH, pos);
    if (tid == 0 && n0 > 0) {         // values of chunk 0 -> buf1
        mbar_expect_tx(&bars[1], (uint32_t)(n0 * hd * (int)sizeof(T)));
        bulk_g2s(buf1, vt, (uint32_t)(n0 * hd * sizeof(T)), &bars[1]);
    }
    if (n0 > 0) load_k_chunk(buf0, kt, a.kstride, 0, n0, hd, CH);   // keys of chunk 0 -> buf0 (async)
    EMB_PROBE(4, 1);
    pdl_wait_then_release();
    EMB_PROBE(4, 2);

    // ---- this position: q, k, v; QK-norm; RoPE; KV store ----
    if (tid < hd) {
        qs[tid] = a.q[h * hd + tid];
        ks[tid] = a.k[kvh * hd + tid];
        vs[tid] = a.v[kvh * hd + tid];
    }
    __syncthreads();
    EMB_PROBE(4, 3);
    if (a.q_norm) {
        // per-head RMSNorm of q and k, in place (ref src/model.c:386-389); the two
        // sequential sums run on different warps
        if (tid == 0) s_q = rms_scale(chain_sumsq(qs, hd), hd, a.eps);
        else if (tid == 32) s_k = rms_scale(chain_sumsq(ks, hd), hd, a.eps);
        __syncthreads();
        if (tid < hd) {
            qs[tid] = fmul(fmul(qs[tid], s_q), qn_s[tid]);
            ks[tid] = fmul(fmul(ks[tid], s_k), kn_s[tid]);
        }
        __syncthreads();
    }
    EMB_PROBE(4, 4);
    // RoPE (ref src/model.c:66-80) with the host-built cos/sin table
    if (tid < hd / 2) {
        const int ia = a.neox ? tid : 2 * tid, ib = a.neox ? tid + hd / 2 : 2 * tid + 1;
        const float2 cs = cs_s[tid];
        float v0 = qs[ia], v1 = qs[ib];
        qs[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        qs[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
        v0 = ks[ia]; v1 = ks[ib];
        ks[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        ks[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
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
    cp_async_wait_all();   // the keys of chunk 0, copied since before the wait
    __syncthreads();

    EMB_PROBE(4, 5);
    // ---- scores: sc = sum_i q_i*k_i in index order, then * (1/sqrt(hd)) ----
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    for (int c = 0; c < nchunks; c++) {
        const int c0 = c * CH, n = min(CH, pos - c0);
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
            att[c0 + t] = fmul(sc, inv_sqrt);
        }
    }
    // the score at t == pos (keys in registers' smem copy), on a thread that had
    // no position in the last chunk
    const int last_n = nchunks > 0 ? pos - (nchunks - 1) * CH : 0;
    if (tid == last_n % ATTN_THREADS) {
        float sc = 0.0f;
        for (int i = 0; i < hd; i++) sc = fadd(sc, fmul(qs[i], ks[i]));
        att[pos] = fmul(sc, inv_sqrt);
    }
    __syncthreads();
    EMB_PROBE(4, 6);
    // the keys are done: value chunk 1 may stream into buf0 during the softmax
    if (tid == 0 && nchunks > 1) {
        const int n1 = min(CH, pos - CH);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bars[0], (uint32_t)(n1 * hd * (int)sizeof(T)));
        bulk_g2s(buf0, vt + (size_t)CH * hd, (uint32_t)(n1 * hd * sizeof(T)), &bars[0]);
    }

    // ---- softmax (ref src/model.c:57-64): the max is order-free ----
    float tmax = -INFINITY;
    for (int t = tid; t <= pos; t += ATTN_THREADS) tmax = fmaxf(tmax, att[t]);
    tmax = warp_max(tmax);
    if (lane == 0) red[warp] = tmax;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < ATTN_THREADS / 32; w++) m = fmaxf(m, red[w]);
        s_max = m;
    }
    __syncthreads();
    const float mx = s_max;
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = expf_exact(a.ex, tab_s, fsub(att[t], mx));
    __syncthreads();
    // the denominator: the reference's sequential sum over t = 0..pos
    if (tid == 0) s_inv = fdiv(1.0f, chain_sum(0.0f, att, pos + 1));
    __syncthreads();
    const float inv = s_inv;
    for (int t = tid; t <= pos; t += ATTN_THREADS) att[t] = fmul(att[t], inv);
    __syncthreads();

    EMB_PROBE(4, 7);
    // ---- out_i = sum_t w_t * v_t,i, sequential over t (ref src/model.c:252-256) ----
    float o = 0.0f;
    for (int c = 0; c < nchunks; c++) {
        const int c0 = c * CH, n = min(CH, pos - c0);
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
            const int n2 = min(CH, pos - (c + 2) * CH);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            uint64_t *bb = in1 ? &bars[1] : &bars[0];
            mbar_expect_tx(bb, (uint32_t)(n2 * hd * (int)sizeof(T)));
            bulk_g2s(vb, vt + (size_t)(c + 2) * CH * hd, (uint32_t)(n2 * hd * sizeof(T)), bb);
        }
    }
    EMB_PROBE(4, 8);
    if (tid < hd) {
        o = fadd(o, fmul(att[pos], vs[tid]));
        const int gi = h * hd + tid;
        if (a.of) a.of[gi] = o;
        float dq;
        int8_t q = quant_lane(o, &dq);   // hd % 32 == 0: each warp owns one block
        a.oq[gi] = q;
        if (lane == 0) a.od[gi / 32] = dq;
    }
    EMB_PROBE(4, 9);
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
    pdl_wait_then_release();
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

// first index of the strict maximum (ref src/sample.c:114-118); NaN never wins
EMB_DEV void am_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__global__ void __launch_bounds__(256) argmax_advance_kernel(const ArgmaxArgs a) {
    __shared__ float sv[256];
    __shared__ int si[256];
    __shared__ bool last;
    pdl_wait_then_release();
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
        // all -inf/NaN, or a NaN at index 0 (nothing compares greater): the
        // reference's loop keeps index 0
        if (idx == 0x7FFFFFFF || isnan(a.logits[0])) idx = 0;
        a.ctl[CTL_TOK] = idx;
        a.ctl[CTL_POS] += 1;
        if (a.out) a.out[a.ctl[CTL_NOUT]] = idx;
        a.ctl[CTL_NOUT] += 1;
        *a.ticket = 0;
    }
}

// prefill bookkeeping between steps: advance the position
__global__ void advance_kernel(int *ctl) {
    pdl_wait_then_release();
    if (threadIdx.x == 0) ctl[CTL_POS] += 1;
}

}  // namespace emb
