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
#include "attn_decode.cuh"

namespace emb {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_MAX_ROWS = 32;     // rows per tile (SwiGLU: exactly one Q8 block of h)
constexpr int GEMV_MAX_STAGES = 4;

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
        // the split sum's barriers publish x and the squares; IN_RAW needs one here
        float sc = 1.0f;
        if (IN == IN_NORM) {
            __syncthreads();
            EMB_PROBE(PK, 3);
            sc = rms_scale(split_chain_sum<GEMV_THREADS>(sq_s, cols), cols, a.eps);
            EMB_PROBE(PK, 4);
        } else {
            __syncthreads();
        }
        // normalize (x*scale)*w and quantize the activation (ref src/kernels.c:211):
        // eight threads per 32-block, four elements each (each thread normalizes
        // the four it quantizes), every block at once
        for (int base = 0; base < nb * 8; base += GEMV_THREADS) {
            const int q8 = base + tid;
            const bool act = q8 < nb * 8;
            const unsigned mask = __ballot_sync(0xffffffffu, act);
            if (act) {
                const int b = q8 >> 3, sub = q8 & 7;
                float4 v = reinterpret_cast<const float4 *>(xf_s + b * 32)[sub];
                if (IN == IN_NORM) {
                    const float4 w = reinterpret_cast<const float4 *>(nw_s + b * 32)[sub];
                    v.x = fmul(fmul(v.x, sc), w.x);
                    v.y = fmul(fmul(v.y, sc), w.y);
                    v.z = fmul(fmul(v.z, sc), w.z);
                    v.w = fmul(fmul(v.w, sc), w.w);
                    reinterpret_cast<float4 *>(xf_s + b * 32)[sub] = v;   // the fp32 weights' path reads it
                }
                float dq;
                const uint32_t packed = quant_quad(v, mask, &dq);
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
