// persist.cuh — the token step as ONE persistent kernel (sm_100a).
//
// Why. A decode step of these models is ~140 small dependent pieces of work
// (5 per layer), each latency-bound by the exact fp32 chains the reference's
// arithmetic requires. As separate launches every piece pays a launch, a
// prologue and an epilogue, and no weight bytes move while a chain runs. Here
// one cooperative launch of one CTA per SM runs whole greedy runs:
//
//   GEMV CTAs (all but the first n_heads)  own fixed row slices of every matrix
//       and stream their slices of the coming stages into a ring of shared-
//       memory slots by bulk asynchronous copies (TMA) while the current stage
//       runs, so weight traffic never waits on a chain;
//   attention CTAs (one per query head)    prefetch the cached keys and values
//       of the next layer while the GEMV stages run.
//
// Per layer the stages are
//   S1 QKV   RMSNorm(x) + Q8 quant, [wq|wk|wv] rows (+bias)       -> q,k,v
//   S2 ATTN  QK-norm, RoPE, KV store, scores, softmax, P.V, quant -> o (Q8)
//   S3 WO    wo rows, x += .                                       -> x
//   S4 W13   RMSNorm(x) + quant, w1/w3 rows, SiLU(g)*u, quant      -> h (Q8)
//   S5 W2    w2 rows, x += .                                       -> x
// then the final norm + lm_head rows, per-CTA argmax partials, and the pick.
//
// Hand-off between CTAs. A stage's outputs are published as 64-bit words that
// carry the 32-bit value and a 32-bit tag (unique per token step, layer and
// stage) in one store; a consumer polls the words it needs until every tag
// matches. A 64-bit store is single-copy atomic, so value and tag are seen
// together: one L2 round trip per hand-off, no fences on the hot path. Tags
// only grow, so stale words of earlier steps never match. Plain global data
// that crosses CTAs (the KV cache) is written before a fence by its writer and
// read much later through L2 (bulk copies, cp.async.cg).
//
// Every wait is bounded: a poll or mbarrier wait that gives up records its code
// in the state's error word, every other wait sees the error word and gives up
// too, each CTA waits (bounded) for its own copies in flight and returns, and
// the host reports `ember: cuda: ...`.
//
// Arithmetic: every fp32 step is the graph path's (kernels.cuh), in the
// reference's order, built from the same helpers: bit-identical results.
#pragma once

#include "common.cuh"

namespace emb {

constexpr int PT = 480;                 // compute threads per CTA (warps 0-14)
constexpr int PNW = PT / 32;
constexpr int PTT = PT + 32;            // + one producer warp (GEMV CTAs: issues the weight copies)

// barriers among the compute threads only (named barrier 1), so that the
// producer warp never takes part
EMB_DEV void csync() { asm volatile("bar.sync 1, 480;" ::: "memory"); }
EMB_DEV bool csync_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\t"
        "setp.ne.u32 a, %1, 0;\n\t"
        "bar.red.or.pred b, 1, 480, a;\n\t"
        "selp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p)
        : "memory");
    return r != 0;
}
constexpr int P_NSLOT = 4;              // weight ring slots per GEMV CTA
constexpr int P_SLOT = 36864;           // bytes per slot
constexpr int P_MAXPIECES = 96;         // pieces of one stage per CTA (lm_head is the longest)
constexpr int P_MAXROWS = 64;           // rows of one piece (w1/w3 pairs: 2 x 32)

enum { PS_QKV = 0, PS_WO = 1, PS_W13 = 2, PS_W2 = 3, PS_HEAD = 4, PS_N = 5 };
// tag offsets within a token step: layer l, stage s -> base + 8 l + s
enum { TG_QKV = 0, TG_O = 1, TG_XA = 2, TG_H = 3, TG_XB = 4 };
constexpr int CTL_TAG = 5;              // ctl word: the next token step's tag base

// per-layer weight pointers in device memory (one entry per layer)
struct PLayer {
    const uint8_t *q[7];     // wq, wk, wv, wo, w1, w2, w3: quantized rows
    const __half *s[7];      //   ... and their fp16 block scales
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm, *bq, *bk, *bv;
};
enum { W_Q = 0, W_K = 1, W_V = 2, W_O = 3, W_1 = 4, W_2 = 5, W_3 = 6 };
constexpr int P_MAXL = 48;              // layers the shared-memory pointer table holds

// the per-layer pointers, copied into shared memory at the start of a launch so
// that no stage waits on a global load for a pointer
__shared__ PLayer p_layers[P_MAXL];

// the dynamic shared memory of the persistent kernel. Every shared-memory
// pointer of the step is derived from this symbol (never mixed with a null or
// global pointer), so the compiler keeps shared-space loads and stores, which
// are several times faster than generic ones.
extern __shared__ __align__(128) unsigned char p_dyn[];

// 4-byte global -> shared copy that completes asynchronously (cp.async); the
// issuing thread waits for its groups with cp.async.wait_group
EMB_DEV void cp_async4(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}

struct PArgs {
    const PLayer *layers;
    const uint8_t *emb_q;      // Q8_0 embedding rows (int8) and scales
    const __half *emb_s;
    const uint8_t *head_q;     // lm_head rows and scales (the embedding when tied)
    const __half *head_s;
    int head_dtype;
    const float *final_norm;
    int wdtype;                // layer matrices: Q8_0 or Q4_0 (all alike)
    int dim, hidden, L, nh, nkv, hd, vocab, ctx, kstride, neox, qk_norm, has_bias, kv16;
    float eps;
    int n_att;                 // attention CTAs (= nh); GEMV CTAs = gridDim.x - n_att
    // KV cache, RoPE table, outputs
    void *kc, *vc;
    size_t k_layer_elems, v_layer_elems;
    const float2 *rope;
    float *logits;
    int *ctl;
    int *out_tokens;           // greedy: the picks go here (NULL: one forward step)
    // tagged hand-off words
    unsigned long long *w_qkv;   // [qd + 2 kvd] fp32 bits
    unsigned long long *w_o;     // [qd/4] packed int8, then [qd/32] fp32 scales
    unsigned long long *w_x;     // [2][dim] fp32 bits (A after wo, B after w2)
    unsigned long long *w_h;     // [hidden/4] packed int8, then [hidden/32] scales
    unsigned long long *w_am;    // [2 * GEMV CTAs] argmax partials (value, index)
    int n_steps;
    uint32_t spin_limit;       // polls before a hand-off wait gives up
    uint32_t poll_ns;          // pause between polls of a hand-off word
    // attention shared-memory plan
    int kcap;                  // cached positions the key region holds ([hd][kcap])
    int vcap0;                 // positions the value region holds
    size_t k_bytes, v_off;     // key region bytes; value region offset
    size_t att_off;            // scores offset (ctx rounded up to 64 floats)
    // GEMV shared-memory plan (offsets into dynamic shared memory)
    size_t g_xf, g_sq, g_xq, g_xd, g_p, g_rowsum, g_h, g_xown, g_nw, g_bias;
    int rp_qkv, rp_wo, rp_w2, rp_head;   // rows per piece
    int pp_w13;                          // w1/w3 pairs per piece (divides 32)
    ExpfDev ex;
};

// Phase probes of the profiling build (-DEMBER_PROBES; compiled out otherwise):
// thread 0 of the first and last GEMV CTA and of the first and last attention
// CTA records the global timer at each stage boundary of one token step.
#ifdef EMBER_PROBES
__device__ unsigned long long g_pp[4][P_MAXL + 1][16];
#define PPROBE(role, l, ev)                                                                 \
    do {                                                                                    \
        if (threadIdx.x == 0 && (role) >= 0 && probe_on) g_pp[role][l][ev] = probe_now(); \
    } while (0)
// finer probes inside one S1 stage and one norm (layer 1, first GEMV CTA)
__shared__ int p_detail;
#define PDETAIL(ev)                                                                  \
    do {                                                                             \
        if (threadIdx.x == 0 && p_detail) g_pp[0][P_MAXL][ev] = probe_now();          \
    } while (0)
#else
#define PPROBE(role, l, ev) \
    do {                    \
    } while (0)
#define PDETAIL(ev) \
    do {            \
    } while (0)
#endif

// ---- the sequential sum of non-negative terms, for 512 threads -------------------
// sum = ((0 + v[0]) + v[1]) + ... + v[n-1] in index order, the reference's loop,
// evaluated as split_chain_sum (common.cuh) does -- K segments; each later
// segment added by NC threads from the NC consecutive floats centred on an
// estimate of the sum before it; the boundaries walked in order, taking the
// chain that started from the sum actually reached, and the rest added
// sequentially where a sum falls outside its window -- sized for a 512-thread
// CTA (480 compute threads): up to 16 segments, each estimated by one warp as a float tree sum (any
// fixed order serves: the estimate only centres the windows). Exact by
// construction; only the time depends on the windows. v: shared memory,
// 16-byte aligned, n a multiple of 16 K. Called by every thread of the CTA.
template <int K, int NC>
EMB_DEV float psum_split(const float *v, int n) {
    constexpr int NB = K - 1;
    static_assert(NB * NC + 1 <= PT && NB <= PNW, "psum_split: too many chains");
    __shared__ float p_seg[K];
    __shared__ uint32_t p_b0[NB];
    __shared__ int p_fin;
    __shared__ float p_cand[NB][NC];
    __shared__ float p_first, p_answer;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m = n / K;
    if (warp < NB) {
        float e = 0.0f;
        for (int i = lane; i < m; i += 32) e = __fadd_rn(e, v[warp * m + i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, o));
        if (lane == 0) p_seg[warp] = e;
    }
    csync();
    // warp 0: running sums of the segments, the window starts
    if (warp == 0) {
        float run = lane < NB ? p_seg[lane] : 0.0f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float up = __shfl_up_sync(0xffffffffu, run, o);
            if (lane >= o) run = __fadd_rn(run, up);
        }
        const uint32_t bc = __float_as_uint(run);
        const bool fin = bc < 0x7F000000u;
        if (lane < NB) p_b0[lane] = bc > NC / 2 ? bc - NC / 2 : 0u;
        const unsigned ok = __ballot_sync(0xffffffffu, fin || lane >= NB);
        if (lane == 0) p_fin = ok == 0xffffffffu;
    }
    csync();
    if (tid <= NC * NB) {
        const bool is_first = tid == NC * NB;
        const int kk = is_first ? 0 : tid / NC, j = tid % NC;
        float s = is_first ? 0.0f : __uint_as_float(p_b0[kk] + (uint32_t)j);
        const float4 *src = reinterpret_cast<const float4 *>(v + (is_first ? 0 : (kk + 1) * m));
        const int q = m / 4;
        float4 c0 = src[0], c1 = src[1], c2 = src[2], c3 = src[3];
#define EMB_ADD4(c)                                                       \
    s = __fadd_rn(s, c.x); s = __fadd_rn(s, c.y); s = __fadd_rn(s, c.z); \
    s = __fadd_rn(s, c.w);
        for (int k = 4; k < q; k += 4) {
            const float4 n0 = src[k], n1 = src[k + 1], n2 = src[k + 2], n3 = src[k + 3];
            EMB_ADD4(c0) EMB_ADD4(c1) EMB_ADD4(c2) EMB_ADD4(c3)
            c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        }
        EMB_ADD4(c0) EMB_ADD4(c1) EMB_ADD4(c2) EMB_ADD4(c3)
#undef EMB_ADD4
        if (is_first) p_first = s;
        else p_cand[kk][j] = s;
    }
    csync();
    float s = p_first;
    int done = 1;
    const bool fin = p_fin != 0;
#pragma unroll
    for (int k = 0; k < NB; k++) {
        const uint32_t jk = __float_as_uint(s) - p_b0[k];
        if (done == k + 1 && fin && jk < (uint32_t)NC) {
            s = p_cand[k][jk];
            done = k + 2;
        }
    }
    if (done == K) return s;
    if (tid == 0) p_answer = chain_sum(s, v + done * m, n - done * m);
    csync();
    return p_answer;
}

// the sum in index order of n non-negative shared-memory terms (n a multiple of
// 16; 16-byte aligned): the most segments that divide it
EMB_DEV float psum(const float *v, int n) {
    if (n % 256 == 0 && n >= 2048) return psum_split<16, 28>(v, n);
    if (n % 128 == 0 && n >= 256) return psum_split<8, 64>(v, n);
    if (n % 64 == 0 && n >= 128) return psum_split<4, 64>(v, n);
    __shared__ float p_small;
    csync();
    if (threadIdx.x == 0) p_small = chain_sum(0.0f, v, n);
    csync();
    return p_small;
}

// sum = ((0 + v[0]) + v[1]) + ... in index order, the next eight terms loaded
// while the current eight are added (v: shared memory, any alignment)
EMB_DEV float pchain(const float *v, int n) {
    float s = 0.0f;
    int i = 0;
    if (n >= 8) {
        float a[8], b[8];
#pragma unroll
        for (int j = 0; j < 8; j++) a[j] = v[j];
        for (i = 8; i + 8 <= n; i += 8) {
#pragma unroll
            for (int j = 0; j < 8; j++) b[j] = v[i + j];
#pragma unroll
            for (int j = 0; j < 8; j++) s = __fadd_rn(s, a[j]);
#pragma unroll
            for (int j = 0; j < 8; j++) a[j] = b[j];
        }
#pragma unroll
        for (int j = 0; j < 8; j++) s = __fadd_rn(s, a[j]);
    }
    for (; i < n; i++) s = __fadd_rn(s, v[i]);
    return s;
}

// ---- tagged words ---------------------------------------------------------------
EMB_DEV void tw_store(unsigned long long *p, uint32_t v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | v;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
EMB_DEV unsigned long long tw_load(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
EMB_DEV int ld_err(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// error codes of the persistent step (the state's error word)
enum { ERR_P_HANDOFF = 11, ERR_P_RING = 12, ERR_P_ATTN = 13 };

// Wait until words src[i] for i = threadIdx.x + j*PT < n all carry `tag`; their
// values go to vals[j]. Every thread calls it (threads past n wait for nothing);
// returns false for the whole CTA when a wait gave up or another CTA reported
// an error.
template <int MAXW>
EMB_DEV bool tw_wait(uint32_t (&vals)[MAXW], const unsigned long long *src, int n, uint32_t tag, const PArgs &a) {
    int *err = a.ctl + CTL_ERR;
    unsigned missing = 0;
#pragma unroll
    for (int j = 0; j < MAXW; j++)
        if ((int)threadIdx.x + j * PT < n) missing |= 1u << j;
    bool fail = false;
    for (uint32_t it = 0; missing; it++) {
        unsigned long long w[MAXW];
#pragma unroll
        for (int j = 0; j < MAXW; j++)
            if (missing >> j & 1u) w[j] = tw_load(src + threadIdx.x + j * PT);
#pragma unroll
        for (int j = 0; j < MAXW; j++)
            if ((missing >> j & 1u) && (uint32_t)(w[j] >> 32) == tag) {
                vals[j] = (uint32_t)w[j];
                missing &= ~(1u << j);
            }
        if (missing && (it & 31u) == 31u) {
            if (ld_err(err) != 0) { fail = true; break; }
            if (it >= a.spin_limit) {
                atomicExch(err, ERR_P_HANDOFF);
                fail = true;
                break;
            }
        }
        if (missing && a.poll_ns) __nanosleep(a.poll_ns);
    }
    return !csync_or(fail);
}

// Wait until the word at p (when not null) carries `tag`; its value to *val.
// Collective over the CTA, like tw_wait.
EMB_DEV bool tw_wait1(uint32_t *val, const unsigned long long *p, uint32_t tag, const PArgs &a) {
    int *err = a.ctl + CTL_ERR;
    bool fail = false;
    if (p) {
        for (uint32_t it = 0;; it++) {
            const unsigned long long w = tw_load(p);
            if ((uint32_t)(w >> 32) == tag) { *val = (uint32_t)w; break; }
            if ((it & 31u) == 31u) {
                if (ld_err(err) != 0) { fail = true; break; }
                if (it >= a.spin_limit) { atomicExch(err, ERR_P_HANDOFF); fail = true; break; }
            }
            if (a.poll_ns) __nanosleep(a.poll_ns);
        }
    }
    return !csync_or(fail);
}

// ---- weight pieces ---------------------------------------------------------------
// A piece is a run of consecutive rows of one matrix (two matrices for w1/w3:
// the same rows of each), copied into one ring slot: the quant rows, then the
// fp16 scale rows from the 16-byte boundary at or below their start (the scale
// arrays are padded on the device, so the rounded copy stays in bounds).
struct Piece {
    int mat;        // W_* of the layer, or -1 for lm_head
    int row0, nrows;
    int out0;       // first output index (row in the stage's concatenated order)
};

struct PieceTab {
    int n[PS_N], first[PS_N];
    Piece p[P_MAXPIECES * 2];
};

// rows [r0, r1) of the stage's concatenated outputs as pieces of <= rp rows,
// split at matrix boundaries; returns the number written
EMB_DEV int cut_pieces(Piece *out, int r0, int r1, int rp, const int *mats, const int *rows, int nmat) {
    int n = 0, base = 0;
    for (int k = 0; k < nmat; k++) {
        const int lo = max(r0, base), hi = min(r1, base + rows[k]);
        for (int r = lo; r < hi; r += rp) {
            Piece pc;
            pc.mat = mats[k];
            pc.row0 = r - base;
            pc.nrows = min(rp, hi - r);
            pc.out0 = r;
            out[n++] = pc;
        }
        base += rows[k];
    }
    return n;
}

}  // namespace emb

namespace emb {

// ---- the GEMV CTA's weight ring -------------------------------------------------
// Slot k % P_NSLOT holds piece k of the CTA's piece sequence: per token step,
// per layer the QKV, WO, W13 and W2 pieces, then the lm_head pieces. One lane
// of the producer warp issues piece k into its slot as soon as the 15 compute
// warps have released piece k - P_NSLOT (each arrives on the slot's `empty`
// barrier once it is past the slot); the compute warps wait on `full`.
struct Cursor {
    int step, l, s, i;
};

struct GShared {
    uint64_t full[P_NSLOT];
    uint64_t empty[P_NSLOT];
    float bv;                  // lm_head argmax partial of this CTA
    int bi, nan0;
    int tok;
};

// quant row bytes of one row of a `cols`-wide matrix
EMB_DEV int p_qrb(int dtype, int cols) { return dtype == EMBER_DT_Q4_0 ? cols / 2 : cols; }

// the 16-byte-aligned window of fp16 scales of rows [row0, row0 + nrows):
// its start (to *src), the bytes from there to the first scale (*skip), and
// its size rounded up to 16 bytes
EMB_DEV uint32_t scale_window(const __half *s, int row0, int nrows, int nb, const unsigned char **src, uint32_t *skip) {
    const uintptr_t sb = (uintptr_t)(s + (size_t)row0 * nb);
    const uintptr_t sb0 = sb & ~(uintptr_t)15;
    *src = reinterpret_cast<const unsigned char *>(sb0);
    *skip = (uint32_t)(sb - sb0);
    return (uint32_t)((sb - sb0 + (size_t)nrows * nb * 2 + 15) & ~(size_t)15);
}

// which stage comes after `c` in the piece sequence (stages without pieces skipped)
EMB_DEV void cursor_next_stage(Cursor &c, const PieceTab &t, int L) {
    for (;;) {
        if (c.s == PS_HEAD) { c.step++; c.l = 0; c.s = PS_QKV; }
        else if (c.s == PS_W2) { c.l++; c.s = c.l == L ? PS_HEAD : PS_QKV; }
        else c.s++;
        c.i = 0;
        if (t.n[c.s] > 0) return;
    }
}

// matrix pointers and column count of a piece
EMB_DEV void piece_mat(const PArgs &a, int l, int mat, const uint8_t **q, const __half **s, int *cols, int *dtype) {
    if (mat < 0) {
        *q = a.head_q; *s = a.head_s; *cols = a.dim; *dtype = a.head_dtype;
        return;
    }
    const PLayer *L = p_layers + l;
    *q = L->q[mat];
    *s = L->s[mat];
    *dtype = a.wdtype;
    *cols = mat == W_O ? a.nh * a.hd : (mat == W_2 ? a.hidden : a.dim);
}

// bulk-copy the piece at cursor c into `slot`, completing on `bar` (slot
// layout: quant rows of A [of B], then A's [and B's] scale window)
EMB_DEV void issue_piece(const PArgs &a, const PieceTab &t, const Cursor &c, unsigned char *slot, uint64_t *bar) {
    const Piece &pc = t.p[t.first[c.s] + c.i];
    const uint8_t *q;
    const __half *s;
    int cols, dtype;
    piece_mat(a, c.l, pc.mat, &q, &s, &cols, &dtype);
    const int nb = cols / 32, qrb = p_qrb(dtype, cols);
    const uint32_t qbytes = (uint32_t)(pc.nrows * qrb);
    const unsigned char *sa_src;
    uint32_t skip;
    const uint32_t sa_bytes = scale_window(s, pc.row0, pc.nrows, nb, &sa_src, &skip);
    if (c.s == PS_W13) {
        const uint8_t *q3;
        const __half *s3;
        piece_mat(a, c.l, W_3, &q3, &s3, &cols, &dtype);
        const unsigned char *sb_src;
        uint32_t skip3;
        const uint32_t sb_bytes = scale_window(s3, pc.row0, pc.nrows, nb, &sb_src, &skip3);
        mbar_expect_tx(bar, 2 * qbytes + sa_bytes + sb_bytes);
        bulk_g2s(slot, q + (size_t)pc.row0 * qrb, qbytes, bar);
        bulk_g2s(slot + qbytes, q3 + (size_t)pc.row0 * qrb, qbytes, bar);
        bulk_g2s(slot + 2 * qbytes, sa_src, sa_bytes, bar);
        bulk_g2s(slot + 2 * qbytes + sa_bytes, sb_src, sb_bytes, bar);
    } else {
        mbar_expect_tx(bar, qbytes + sa_bytes);
        bulk_g2s(slot, q + (size_t)pc.row0 * qrb, qbytes, bar);
        bulk_g2s(slot + qbytes, sa_src, sa_bytes, bar);
    }
}

// bounded wait on an mbarrier phase that gives up early when the error word is set
EMB_DEV bool mbar_wait_err(uint64_t *bar, uint32_t parity, const PArgs &a, int code) {
    uint32_t i = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++i & 255u) == 0) {
            if (ld_err(a.ctl + CTL_ERR) != 0) return false;
            if (i >= MBAR_TRIES) {
                atomicExch(a.ctl + CTL_ERR, code);
                return false;
            }
        }
    }
    return true;
}

// The producer (lane 0 of warp 15): every piece of the launch in order, each
// once its slot is released. On an error it stops issuing and waits (bounded)
// for the copies it has in flight before the CTA leaves.
EMB_DEV void ring_producer(const PArgs &a, const PieceTab &t, GShared &g, unsigned char *ring) {
    Cursor c;
    c.step = 0; c.l = 0; c.s = PS_QKV; c.i = 0;
    if (t.n[PS_QKV] == 0) cursor_next_stage(c, t, a.L);
    unsigned k = 0;
    for (; c.step < a.n_steps; k++) {
        const int slot = (int)(k % P_NSLOT);
        if (k >= (unsigned)P_NSLOT && !mbar_wait_err(&g.empty[slot], ((k / P_NSLOT) - 1) & 1u, a, ERR_P_RING)) break;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_piece(a, t, c, ring + (size_t)slot * P_SLOT, &g.full[slot]);
        if (++c.i >= t.n[c.s]) cursor_next_stage(c, t, a.L);
    }
    for (unsigned j = k > (unsigned)P_NSLOT ? k - P_NSLOT : 0; j < k; j++)
        for (uint32_t i = 0; i < MBAR_TRIES; i++)
            if (mbar_try_wait(&g.full[j % P_NSLOT], (j / P_NSLOT) & 1u)) break;
}

// Compute threads: wait for piece k (one lane per warp) and agree on the
// outcome; false when a wait gave up or another CTA reported an error. The
// piece is in slot k % P_NSLOT of the ring at the start of p_dyn.
EMB_DEV bool ring_acquire(const PArgs &a, GShared &g, unsigned k) {
    const int slot = (int)(k % P_NSLOT);
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_err(&g.full[slot], (k / P_NSLOT) & 1u, a, ERR_P_RING);
    __syncwarp();
    return !csync_or(!ok);
}

// a warp is past piece k's slot: its arrival on the slot's `empty` barrier
EMB_DEV void ring_release(GShared &g, unsigned k) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&g.empty[k % P_NSLOT]);
}

// ---- activations in -----------------------------------------------------------------
// x (dim fp32) from the tagged words into xf
EMB_DEV bool gather_x(const PArgs &a, float *xf, const unsigned long long *src, uint32_t tag) {
    uint32_t v[4];
    if (!tw_wait<4>(v, src, a.dim, tag, a)) return false;
#pragma unroll
    for (int j = 0; j < 4; j++)
        if ((int)threadIdx.x + j * PT < a.dim) xf[threadIdx.x + j * PT] = __uint_as_float(v[j]);
    csync();
    return true;
}

// a Q8 activation of n elements (n/4 packed words, then n/32 scale words)
EMB_DEV bool gather_q8(const PArgs &a, int8_t *xq, float *xd, const unsigned long long *src, int n, uint32_t tag) {
    uint32_t v[4];
    const int nw = n / 4 + n / 32;
    if (!tw_wait<4>(v, src, nw, tag, a)) return false;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int i = (int)threadIdx.x + j * PT;
        if (i < n / 4) reinterpret_cast<uint32_t *>(xq)[i] = v[j];
        else if (i < nw) xd[i - n / 4] = __uint_as_float(v[j]);
    }
    csync();
    return true;
}

// RMSNorm of xf in place (ref src/model.c:50-55: the sum of squares in index
// order, 1/sqrtf(ss/n + eps), (x*scale)*w), then the Q8_0 quantization of every
// block into xq / xd (ref src/kernels.c:73-92). w_s: the norm weights in shared
// memory, copied there by this CTA's cp.async group before the newest one.
EMB_DEV void norm_quant(const PArgs &a, float *xf, float *sq, int8_t *xq, float *xd, const float *w_s) {
    const int n = a.dim, nb = n / 32;
    PDETAIL(6);
    cp_async_wait_1();
    for (int i = threadIdx.x; i < n; i += PT) sq[i] = fmul(xf[i], xf[i]);
    csync();
    PDETAIL(7);
    const float sc = rms_scale(psum(sq, n), n, a.eps);
    PDETAIL(8);
    for (int i = threadIdx.x; i < n; i += PT) xf[i] = fmul(fmul(xf[i], sc), w_s[i]);
    csync();
    PDETAIL(9);
    for (int base = 0; base < nb * 8; base += PT) {
        const int q8 = base + (int)threadIdx.x;
        const bool act = q8 < nb * 8;
        const unsigned mask = __ballot_sync(0xffffffffu, act);
        if (act) {
            const int b = q8 >> 3, sub = q8 & 7;
            float dq;
            const uint32_t packed = quant_quad(reinterpret_cast<const float4 *>(xf + b * 32)[sub], mask, &dq);
            reinterpret_cast<uint32_t *>(xq + b * 32)[sub] = packed;
            if (sub == 0) xd[b] = dq;
        }
    }
    csync();
    PDETAIL(10);
}

}  // namespace emb

namespace emb {

// shared-memory views of a GEMV CTA
struct GViews {
    unsigned char *ring;
    float *xf, *sq, *xd, *P, *rowsum, *hbuf, *xown;
    float *nw;                 // norm weights, two layers: [buffer][attn, ffn][dim]
    float *bias;               // this layer's q/k/v biases of this CTA's S1 rows
    int8_t *xq;
    double *tab;
    int own0, own1;            // x rows this CTA owns (wo / w2 outputs)
    int qkv0;                  // first S1 row of this CTA
};

EMB_DEV bool am_better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// The Q8_0 terms of the rows of one piece, NSP 512-byte spans per row, fully
// unrolled for the compiler: warp w takes rows w, w + 15, ... (RPW of them:
// rows <= 15 RPW), lane l the 16 bytes [16 l, 16 l + 16) of each span, so all loads can be
// in flight at once. x4 / dx: this lane's activation bytes and block scale per
// span (read from the activation in shared memory, xq / xd). Row rr's weights
// are at wq(rr), its fp16 scales at ws(rr), its terms go to P + rr * pstride.
template <int NSP, int RPW, typename WQ, typename WS>
EMB_DEV void dots_q8(const WQ &wq, const WS &ws, float *P, int pstride, int rows, int cols, const int8_t *xq,
                     const float *xd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int4 x4[NSP];
    float dx[NSP];
#pragma unroll
    for (int sp = 0; sp < NSP; sp++) {
        const int off = sp * 512 + lane * 16;
        x4[sp] = off < cols ? *reinterpret_cast<const int4 *>(xq + off) : make_int4(0, 0, 0, 0);
        dx[sp] = off < cols ? xd[off / 32] : 0.0f;
    }
    int acc[RPW][NSP];
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const int rr = warp + k * PNW;
        const uint8_t *w = wq(rr < rows ? rr : 0);
#pragma unroll
        for (int sp = 0; sp < NSP; sp++) {
            const int off = sp * 512 + lane * 16;
            int a = 0;
            if (off < cols) {
                const int4 w4 = *reinterpret_cast<const int4 *>(w + off);
                a = __dp4a(w4.x, x4[sp].x, a); a = __dp4a(w4.y, x4[sp].y, a);
                a = __dp4a(w4.z, x4[sp].z, a); a = __dp4a(w4.w, x4[sp].w, a);
            }
            acc[k][sp] = a;
        }
    }
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const int rr = warp + k * PNW;
        const __half *s = ws(rr < rows ? rr : 0);
#pragma unroll
        for (int sp = 0; sp < NSP; sp++) {
            const int off = sp * 512 + lane * 16;
            const int a = acc[k][sp] + __shfl_xor_sync(0xffffffffu, acc[k][sp], 1);
            if (rr < rows && off < cols && (lane & 1) == 0) {
                const int b = off / 32;
                P[rr * pstride + b] = fmul(fmul(__int2float_rn(a), __half2float(s[b])), dx[sp]);
            }
        }
    }
}

// One stage of a GEMV CTA over its pieces of layer l. Per piece: each warp takes
// rows (warp w: rows w, w+15, ...) and forms the terms ((float)acc * d_w) * d_x
// of every block of the row in shared memory -- Q8_0 rows in 512-byte spans,
// lane l reading bytes [16 l, 16 l + 16) of the span (contiguous across the
// warp, so without bank conflicts) against the matching activation bytes held
// in registers, the two lanes of a block joined by one shuffle (the int32 block
// sum is exact in any order); Q4_0 rows a block per lane -- then releases the
// slot; then one lane per row adds the row's terms in block order (ref
// src/kernels.c:152-164) and runs the stage's epilogue. The activation (xq, xd)
// is in shared memory already; kc counts the pieces consumed.
template <int ST>
EMB_DEV bool gemv_stage(const PArgs &a, const PieceTab &t, GShared &g, const GViews &v, int l, uint32_t tag,
                        unsigned &kc) {
    constexpr int nsub = ST == PS_W13 ? 2 : 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const PLayer *Lp = p_layers + l;
    float hb_v = -INFINITY;    // HEAD: this lane's best logit so far, and its index
    int hb_i = 0x7FFFFFFF;
    for (int i = 0; i < t.n[ST]; i++) {
        const Piece pc = t.p[t.first[ST] + i];
        if (ST == PS_QKV && i == 0) PDETAIL(0);
        if (!ring_acquire(a, g, kc)) return false;
        const unsigned char *slot = p_dyn + (size_t)(kc % P_NSLOT) * P_SLOT;
        if (ST == PS_QKV && i == 0) PDETAIL(1);
        const uint8_t *q;
        const __half *s;
        int cols, dtype;
        piece_mat(a, l, pc.mat, &q, &s, &cols, &dtype);
        const int nb = cols / 32, qrb = p_qrb(dtype, cols), pstride = nb | 1, nr = pc.nrows;
        const uint32_t qbytes = (uint32_t)(nr * qrb);
        const unsigned char *src;
        uint32_t skip_a, skip_b = 0;
        const uint32_t sa_bytes = scale_window(s, pc.row0, nr, nb, &src, &skip_a);
        const __half *sc_a = reinterpret_cast<const __half *>(slot + nsub * qbytes + skip_a);
        const __half *sc_b = sc_a;
        if (ST == PS_W13) {
            scale_window(Lp->s[W_3], pc.row0, nr, nb, &src, &skip_b);
            sc_b = reinterpret_cast<const __half *>(slot + 2 * qbytes + sa_bytes + skip_b);
        }
        const int rows = nsub * nr;
#ifdef EMBER_PROBES
        // profiling build: the first S1 piece's dot loop runs twice (the same
        // instructions), to time it cold and warm
        const int reps = (ST == PS_QKV && i == 0 && p_detail) ? 2 : 1;
        for (int rep = 0; rep < reps; rep++) {
        if (rep == 1) { csync(); PDETAIL(11); }
#endif
        if (dtype == EMBER_DT_Q8_0) {
            const int nsp = (cols + 511) / 512;
            auto wq = [&](int rr) {
                const int sub = nsub == 2 && rr >= nr ? 1 : 0;
                return slot + sub * qbytes + (size_t)(rr - sub * nr) * qrb;
            };
            auto wsf = [&](int rr) {
                const int sub = nsub == 2 && rr >= nr ? 1 : 0;
                return (sub ? sc_b : sc_a) + (rr - sub * nr) * nb;
            };
            if (nsp <= 2 && rows <= 3 * PNW) {
                dots_q8<2, 3>(wq, wsf, v.P, pstride, rows, cols, v.xq, v.xd);
            } else if (nsp <= 4 && rows <= 2 * PNW) {
                dots_q8<4, 2>(wq, wsf, v.P, pstride, rows, cols, v.xq, v.xd);
            } else if (nsp <= 6 && rows <= PNW) {
                dots_q8<6, 1>(wq, wsf, v.P, pstride, rows, cols, v.xq, v.xd);
            } else {
                // wider rows or taller pieces: span by span, a row at a time
                for (int rr = warp; rr < rows; rr += PNW) {
                    const uint8_t *w = wq(rr);
                    const __half *sc = wsf(rr);
                    for (int sp = 0; sp < nsp; sp++) {
                        const int off = sp * 512 + lane * 16;
                        const int4 x4 = off < cols ? *reinterpret_cast<const int4 *>(v.xq + off) : make_int4(0, 0, 0, 0);
                        int acc = 0;
                        if (off < cols) {
                            const int4 w4 = *reinterpret_cast<const int4 *>(w + off);
                            acc = __dp4a(w4.x, x4.x, acc); acc = __dp4a(w4.y, x4.y, acc);
                            acc = __dp4a(w4.z, x4.z, acc); acc = __dp4a(w4.w, x4.w, acc);
                        }
                        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                        if (off < cols && (lane & 1) == 0) {
                            const int bk = off / 32;
                            v.P[rr * pstride + bk] = fmul(fmul(__int2float_rn(acc), __half2float(sc[bk])), v.xd[bk]);
                        }
                    }
                }
            }
        } else {
            for (int rr = warp; rr < rows; rr += PNW) {
                const int sub = nsub == 2 && rr >= nr ? 1 : 0, r = rr - sub * nr;
                const uint8_t *wq = slot + sub * qbytes + (size_t)r * qrb;
                const __half *ws = (sub ? sc_b : sc_a) + r * nb;
                float *pr = v.P + rr * pstride;
                for (int b = lane; b < nb; b += 32) {
                    const int acc = dot_q4_block(wq + b * 16, v.xq + b * 32);
                    pr[b] = fmul(fmul(__int2float_rn(acc), __half2float(ws[b])), v.xd[b]);
                }
            }
        }
#ifdef EMBER_PROBES
        if (rep == 0) { csync(); if (ST == PS_QKV && i == 0) PDETAIL(2); }
        }
        if (reps == 2) { csync(); PDETAIL(12); }
#else
        if (ST == PS_QKV && i == 0) PDETAIL(2);
#endif
        ring_release(g, kc);
        kc++;
        csync();
        if (ST == PS_QKV && i == 0) PDETAIL(3);
        // chains and epilogue: row rr = warp + 15 * lane on lanes 0..4
        const int rr = warp + PNW * lane;
        if (lane < 5 && rr < rows) {
            const float y = pchain(v.P + rr * pstride, nb);
            if (ST == PS_QKV) {
                float o = y;
                if (a.has_bias) o = fadd(o, v.bias[pc.out0 + rr - v.qkv0]);   // ref src/model.c:382-384
                tw_store(a.w_qkv + pc.out0 + rr, __float_as_uint(o), tag);
            } else if (ST == PS_WO || ST == PS_W2) {
                const int row = pc.out0 + rr;
                const float xn = fadd(v.xown[row - v.own0], y);   // x += y (ref :398, :408)
                v.xown[row - v.own0] = xn;
                tw_store(a.w_x + (ST == PS_W2 ? a.dim : 0) + row, __float_as_uint(xn), tag);
            } else if (ST == PS_W13) {
                v.rowsum[rr] = y;
            } else {   // PS_HEAD
                const int row = pc.out0 + rr;
                a.logits[row] = y;
                if (row == 0 && !(y == y)) g.nan0 = 1;
                if (y == y && am_better(y, row, hb_v, hb_i)) { hb_v = y; hb_i = row; }   // NaN never wins
            }
        }
        if (ST == PS_QKV && i == 0) PDETAIL(4);
        if (ST == PS_W13) {
            // h = SiLU(g) * u = g / (1 + expf(-g)) * u (ref src/model.c:403-406)
            csync();
            const int in_blk = pc.out0 & 31;
            if (tid < nr) {
                const float gv = v.rowsum[tid], uv = v.rowsum[nr + tid];
                const float e = expf_exact(a.ex, v.tab, -gv);
                v.hbuf[in_blk + tid] = fmul(fdiv(gv, fadd(1.0f, e)), uv);
            }
            if (in_blk + nr == 32) {
                // the block of h is complete: its Q8 quantization for w2, published
                csync();
                if (tid < 32) {
                    float dq;
                    const int8_t qv = quant_lane(v.hbuf[tid], &dq);
                    uint32_t b = (uint32_t)(uint8_t)qv;
                    b |= (uint32_t)__shfl_down_sync(0xffffffffu, b, 1) << 8;
                    b |= (uint32_t)__shfl_down_sync(0xffffffffu, b, 2) << 16;
                    const int blk = pc.out0 >> 5;
                    if ((tid & 3) == 0) tw_store(a.w_h + blk * 8 + tid / 4, b, tag);
                    if (tid == 0) tw_store(a.w_h + a.hidden / 4 + blk, __float_as_uint(dq), tag);
                }
            }
        }
        csync();   // P is written again by the next piece
    }
    if (ST == PS_HEAD) {
        // this CTA's first maximum over all its rows: lanes, then warps
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, hb_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, hb_i, o);
            if (am_better(ov, oi, hb_v, hb_i)) { hb_v = ov; hb_i = oi; }
        }
        __shared__ float h_v[PNW];
        __shared__ int h_i[PNW];
        if (lane == 0) { h_v[warp] = hb_v; h_i[warp] = hb_i; }
        csync();
        if (warp == 0) {
            float bv = lane < PNW ? h_v[lane] : -INFINITY;
            int bi = lane < PNW ? h_i[lane] : 0x7FFFFFFF;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0 && am_better(bv, bi, g.bv, g.bi)) { g.bv = bv; g.bi = bi; }
        }
        csync();
    }
    return true;
}

}  // namespace emb

namespace emb {

// the attention CTA's shared state
struct AShared {
    uint64_t vbar[2];          // values of chunk 0 (value region), chunk 1 (key region)
    uint32_t vph[2];           // their phases
    int pending[2];            // a copy on vbar[i] is in flight
    __align__(16) float qs[256];
    __align__(16) float ks[256];
    __align__(16) float vs[256];
    __align__(16) float qn[256];
    __align__(16) float kn[256];
    __align__(16) float2 cs[128];
    float red[PNW];
    float s_q, s_k, s_max, s_inv;
};

// Start moving layer l's cache for a query at `pos` into shared memory: the keys
// of positions [0, pos) into the transposed key region [hd][kcap] by 16-byte
// cp.async (rows are padded to kstride, so rounding up to a vector stays in
// bounds), the layer's QK-norm weights and this position's cos/sin, and the
// values of [0, min(pos, vcap0)) into the value region by one bulk copy. The
// rest of the values follow into the key region once the scores are done.
template <typename T>
EMB_DEV void attn_prefetch(const PArgs &a, AShared &sh, unsigned char *smem, int l, int pos) {
    const int h = blockIdx.x, kvh = h / (a.nh / a.nkv), hd = a.hd;
    const T *kt = reinterpret_cast<const T *>(a.kc) + (size_t)l * a.k_layer_elems + (size_t)kvh * hd * a.kstride;
    const T *vt = reinterpret_cast<const T *>(a.vc) + (size_t)l * a.v_layer_elems + (size_t)kvh * a.ctx * hd;
    T *kbuf = reinterpret_cast<T *>(smem);
    constexpr int E = 16 / (int)sizeof(T);
    const int nv = (pos + E - 1) / E, total = hd * nv;
    for (int idx = threadIdx.x; idx < total; idx += PT) {
        const int i = idx / nv, vv = idx - i * nv;
        cp_async16(kbuf + (size_t)i * a.kcap + vv * E, kt + (size_t)i * a.kstride + vv * E);
    }
    const PLayer *Lp = p_layers + l;
    for (int i = threadIdx.x; i < hd / 4; i += PT) {
        if (a.qk_norm && Lp->q_norm) {
            cp_async16(sh.qn + 4 * i, Lp->q_norm + 4 * i);
            cp_async16(sh.kn + 4 * i, Lp->k_norm + 4 * i);
        }
        cp_async16(sh.cs + 2 * i, a.rope + (size_t)pos * (hd / 2) + 2 * i);
    }
    cp_async_commit();
    const int n0 = min(pos, a.vcap0);
    if (threadIdx.x == 0 && n0 > 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&sh.vbar[0], (uint32_t)(n0 * hd * sizeof(T)));
        bulk_g2s(smem + a.v_off, vt, (uint32_t)(n0 * hd * sizeof(T)), &sh.vbar[0]);
        sh.pending[0] = 1;
    }
}

// thread 0: bounded wait for the copy on vbar[i] (if one is in flight)
EMB_DEV bool attn_wait_v(const PArgs &a, AShared &sh, int i) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        int ok = 1;
        if (sh.pending[i]) {
            ok = mbar_wait(&sh.vbar[i], sh.vph[i], a.ctl + CTL_ERR, ERR_P_ATTN) ? 1 : 0;
            if (ok) { sh.vph[i] ^= 1u; sh.pending[i] = 0; }
        }
        s_ok = ok;
    }
    csync();
    return s_ok != 0;
}

// S2 of layer l for query head h = blockIdx.x at position pos (ref
// src/model.c:386-398 and :221-259), the arithmetic of attn_decode_kernel.
template <typename T>
EMB_DEV bool attn_stage(const PArgs &a, AShared &sh, unsigned char *smem, const double *tab, int l, int pos,
                        uint32_t tag_in, uint32_t tag_out, int role, bool probe_on) {
    (void)role;
    (void)probe_on;
    PPROBE(role, l, 0);
    const int h = blockIdx.x, tid = threadIdx.x, hd = a.hd, lane = tid & 31, warp = tid >> 5;
    const int kv_mul = a.nh / a.nkv, kvh = h / kv_mul, qd = a.nh * hd, kvd = a.nkv * hd;
    const PLayer *Lp = p_layers + l;
    T *kt = reinterpret_cast<T *>(a.kc) + (size_t)l * a.k_layer_elems + (size_t)kvh * hd * a.kstride;
    T *vt = reinterpret_cast<T *>(a.vc) + (size_t)l * a.v_layer_elems + (size_t)kvh * a.ctx * hd;
    const T *kbuf = reinterpret_cast<const T *>(smem);
    float *att = reinterpret_cast<float *>(smem + a.att_off);
    // the keys, norm weights and cos/sin requested during the previous stages
    cp_async_wait_all();
    // this position's q, k, v from the projection
    {
        const unsigned long long *p = nullptr;
        if (tid < hd) p = a.w_qkv + h * hd + tid;
        else if (tid < 2 * hd) p = a.w_qkv + qd + kvh * hd + (tid - hd);
        else if (tid < 3 * hd) p = a.w_qkv + qd + kvd + kvh * hd + (tid - 2 * hd);
        uint32_t val = 0;
        if (!tw_wait1(&val, p, tag_in, a)) return false;
        if (tid < hd) sh.qs[tid] = __uint_as_float(val);
        else if (tid < 2 * hd) sh.ks[tid - hd] = __uint_as_float(val);
        else if (tid < 3 * hd) sh.vs[tid - 2 * hd] = __uint_as_float(val);
        csync();
    }
    PPROBE(role, l, 1);
    if (a.qk_norm && Lp->q_norm) {
        // per-head RMSNorm of q and k (ref src/model.c:386-389), two chains on two warps
        if (tid == 0) sh.s_q = rms_scale(chain_sumsq(sh.qs, hd), hd, a.eps);
        else if (tid == 32) sh.s_k = rms_scale(chain_sumsq(sh.ks, hd), hd, a.eps);
        csync();
        if (tid < hd) {
            sh.qs[tid] = fmul(fmul(sh.qs[tid], sh.s_q), sh.qn[tid]);
            sh.ks[tid] = fmul(fmul(sh.ks[tid], sh.s_k), sh.kn[tid]);
        }
        csync();
    }
    // RoPE (ref src/model.c:66-80) with the host-built cos/sin table
    if (tid < hd / 2) {
        const int ia = a.neox ? tid : 2 * tid, ib = a.neox ? tid + hd / 2 : 2 * tid + 1;
        const float2 cs = sh.cs[tid];
        float v0 = sh.qs[ia], v1 = sh.qs[ib];
        sh.qs[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        sh.qs[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
        v0 = sh.ks[ia]; v1 = sh.ks[ib];
        sh.ks[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        sh.ks[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
    }
    csync();
    // KV store (ref src/model.c:39-48): attention reads the stored (rounded)
    // values, including at t == pos; the first query head of each kv head writes
    // the cache (and fences after publishing its output, before anything of a
    // later step can read the entry)
    if (tid < hd) {
        T kq, vq;
        kv_round(sh.ks[tid], &kq);
        kv_round(sh.vs[tid], &vq);
        sh.ks[tid] = widen(kq);
        sh.vs[tid] = widen(vq);
        if (h % kv_mul == 0) {
            kt[(size_t)tid * a.kstride + pos] = kq;
            vt[(size_t)pos * hd + tid] = vq;
        }
    }
    csync();
    PPROBE(role, l, 2);
    // scores: sc = sum_i q_i*k_i in index order, then * (1/sqrt(hd))
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    for (int t = tid; t < pos; t += PT) {
        float sc = 0.0f;
        for (int i = 0; i < hd; i += 8) {
            float kk[8];
#pragma unroll
            for (int j = 0; j < 8; j++) kk[j] = widen(kbuf[(size_t)(i + j) * a.kcap + t]);
#pragma unroll
            for (int j = 0; j < 8; j++) sc = fadd(sc, fmul(sh.qs[i + j], kk[j]));
        }
        att[t] = fmul(sc, inv_sqrt);
    }
    if (tid == pos % PT) {
        float sc = 0.0f;
        for (int i = 0; i < hd; i++) sc = fadd(sc, fmul(sh.qs[i], sh.ks[i]));
        att[pos] = fmul(sc, inv_sqrt);
    }
    // zeros after the last score, up to the padded length of the denominator
    const int npad = (pos + 1 + 63) / 64 * 64;
    for (int t = pos + 1 + tid; t < npad; t += PT) att[t] = 0.0f;
    csync();
    PPROBE(role, l, 3);
    // the keys are done: the values past the value region stream into their space
    if (tid == 0 && pos > a.vcap0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t nb1 = (uint32_t)((pos - a.vcap0) * hd * sizeof(T));
        mbar_expect_tx(&sh.vbar[1], nb1);
        bulk_g2s(smem, vt + (size_t)a.vcap0 * hd, nb1, &sh.vbar[1]);
        sh.pending[1] = 1;
    }
    // softmax (ref src/model.c:57-64): the max is order-free
    float tmax = -INFINITY;
    for (int t = tid; t <= pos; t += PT) tmax = fmaxf(tmax, att[t]);
    tmax = warp_max(tmax);
    if (lane == 0) sh.red[warp] = tmax;
    csync();
    if (warp == 0) {
        const float m = warp_max(lane < PNW ? sh.red[lane] : -INFINITY);
        if (lane == 0) sh.s_max = m;
    }
    csync();
    const float mx = sh.s_max;
    for (int t = tid; t <= pos; t += PT) att[t] = expf_exact(a.ex, tab, fsub(att[t], mx));
    csync();
    // the denominator: the reference's sequential sum over t = 0..pos (the zero
    // padding adds nothing)
    const float den = psum(att, npad);
    if (tid == 0) sh.s_inv = fdiv(1.0f, den);
    csync();
    const float inv = sh.s_inv;
    for (int t = tid; t <= pos; t += PT) att[t] = fmul(att[t], inv);
    csync();
    PPROBE(role, l, 4);
    // out_i = sum_t w_t * v_t,i, sequential over t (ref src/model.c:252-256)
    if (!attn_wait_v(a, sh, 0)) return false;
    float o = 0.0f;
    const T *vb0 = reinterpret_cast<const T *>(smem + a.v_off);
    const int n0 = min(pos, a.vcap0);
    if (tid < hd) {
        int t = 0;
        for (; t + 8 <= n0; t += 8) {
            float ww[8], vv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) { ww[j] = att[t + j]; vv[j] = widen(vb0[(size_t)(t + j) * hd + tid]); }
#pragma unroll
            for (int j = 0; j < 8; j++) o = fadd(o, fmul(ww[j], vv[j]));
        }
        for (; t < n0; t++) o = fadd(o, fmul(att[t], widen(vb0[(size_t)t * hd + tid])));
    }
    if (pos > a.vcap0) {
        if (!attn_wait_v(a, sh, 1)) return false;
        const T *vb1 = reinterpret_cast<const T *>(smem);
        if (tid < hd) {
            const int n1 = pos - a.vcap0;
            const float *w1 = att + a.vcap0;
            int t = 0;
            for (; t + 8 <= n1; t += 8) {
                float ww[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) { ww[j] = w1[t + j]; vv[j] = widen(vb1[(size_t)(t + j) * hd + tid]); }
#pragma unroll
                for (int j = 0; j < 8; j++) o = fadd(o, fmul(ww[j], vv[j]));
            }
            for (; t < n1; t++) o = fadd(o, fmul(w1[t], widen(vb1[(size_t)t * hd + tid])));
        }
    }
    if (tid < hd) {
        o = fadd(o, fmul(att[pos], sh.vs[tid]));
        // Q8 quantization of the head output: hd % 32 == 0, one block per warp
        float dq;
        const int8_t qv = quant_lane(o, &dq);
        uint32_t b = (uint32_t)(uint8_t)qv;
        b |= (uint32_t)__shfl_down_sync(0xffffffffu, b, 1) << 8;
        b |= (uint32_t)__shfl_down_sync(0xffffffffu, b, 2) << 16;
        const int gi = h * hd + tid;
        if ((lane & 3) == 0) tw_store(a.w_o + gi / 4, b, tag_out);
        if (lane == 0) tw_store(a.w_o + qd / 4 + gi / 32, __float_as_uint(dq), tag_out);
    }
    PPROBE(role, l, 5);
    // the cache entry written above, ordered before every later hand-off of this
    // CTA (its readers come a step later, behind several of them)
    if (tid < hd && h % kv_mul == 0) __threadfence();
    csync();
    return true;
}

}  // namespace emb

namespace emb {

// tag base of token step `step` of a launch whose first base is T0
EMB_DEV uint32_t step_tag(uint32_t T0, int step, int L) { return T0 + (uint32_t)step * (uint32_t)(8 * L + 8); }

// thread 0: the pieces of every stage for GEMV CTA gi of G
EMB_DEV void build_pieces(const PArgs &a, PieceTab &t, int gi, int G) {
    const int qd = a.nh * a.hd, kvd = a.nkv * a.hd;
    int n = 0;
    {
        const int R = qd + 2 * kvd, mats[3] = {W_Q, W_K, W_V}, rows[3] = {qd, kvd, kvd};
        t.first[PS_QKV] = n;
        n += cut_pieces(t.p + n, (int)((long)gi * R / G), (int)((long)(gi + 1) * R / G), a.rp_qkv, mats, rows, 3);
        t.n[PS_QKV] = n - t.first[PS_QKV];
    }
    const int o0 = (int)((long)gi * a.dim / G), o1 = (int)((long)(gi + 1) * a.dim / G);
    {
        const int mats[1] = {W_O}, rows[1] = {a.dim};
        t.first[PS_WO] = n;
        n += cut_pieces(t.p + n, o0, o1, a.rp_wo, mats, rows, 1);
        t.n[PS_WO] = n - t.first[PS_WO];
    }
    {
        const int NB = a.hidden / 32, b0 = (int)((long)gi * NB / G), b1 = (int)((long)(gi + 1) * NB / G);
        t.first[PS_W13] = n;
        for (int b = b0; b < b1; b++)
            for (int k = 0; k < 32; k += a.pp_w13) {
                Piece pc;
                pc.mat = W_1;
                pc.row0 = b * 32 + k;
                pc.nrows = a.pp_w13;
                pc.out0 = pc.row0;
                t.p[n++] = pc;
            }
        t.n[PS_W13] = n - t.first[PS_W13];
    }
    {
        const int mats[1] = {W_2}, rows[1] = {a.dim};
        t.first[PS_W2] = n;
        n += cut_pieces(t.p + n, o0, o1, a.rp_w2, mats, rows, 1);
        t.n[PS_W2] = n - t.first[PS_W2];
    }
    {
        const int mats[1] = {-1}, rows[1] = {a.vocab};
        t.first[PS_HEAD] = n;
        n += cut_pieces(t.p + n, (int)((long)gi * a.vocab / G), (int)((long)(gi + 1) * a.vocab / G), a.rp_head,
                        mats, rows, 1);
        t.n[PS_HEAD] = n - t.first[PS_HEAD];
    }
}

// x = the token's embedding row, dequantized as q*d (ref src/model.c:83-100)
EMB_DEV void embed_row(const PArgs &a, int tok, float *xf) {
    const int8_t *row = reinterpret_cast<const int8_t *>(a.emb_q) + (size_t)tok * a.dim;
    const __half *sc = a.emb_s + (size_t)tok * (a.dim / 32);
    for (int i = threadIdx.x; i < a.dim; i += PT) xf[i] = fmul((float)row[i], __half2float(sc[i / 32]));
    csync();
}

EMB_DEV bool gemv_cta(const PArgs &a, unsigned char *smem, double *tab, int gi, int G) {
    __shared__ __align__(16) PieceTab t;
    __shared__ __align__(8) GShared g;
    const int tid = threadIdx.x, L = a.L, qd = a.nh * a.hd;
    GViews v;
    v.ring = p_dyn;
    v.xf = reinterpret_cast<float *>(p_dyn + a.g_xf);
    v.sq = reinterpret_cast<float *>(p_dyn + a.g_sq);
    v.xq = reinterpret_cast<int8_t *>(p_dyn + a.g_xq);
    v.xd = reinterpret_cast<float *>(p_dyn + a.g_xd);
    v.P = reinterpret_cast<float *>(p_dyn + a.g_p);
    v.rowsum = reinterpret_cast<float *>(p_dyn + a.g_rowsum);
    v.hbuf = reinterpret_cast<float *>(p_dyn + a.g_h);
    v.xown = reinterpret_cast<float *>(p_dyn + a.g_xown);
    v.nw = reinterpret_cast<float *>(p_dyn + a.g_nw);
    v.bias = reinterpret_cast<float *>(p_dyn + a.g_bias);
    v.tab = tab;
    v.own0 = (int)((long)gi * a.dim / G);
    v.own1 = (int)((long)(gi + 1) * a.dim / G);
    const int R1 = qd + 2 * a.nkv * a.hd;
    v.qkv0 = (int)((long)gi * R1 / G);
    const int qkv1 = (int)((long)(gi + 1) * R1 / G);
    const uint32_t T0 = (uint32_t)a.ctl[CTL_TAG];
    const int pos0 = a.ctl[CTL_POS], nout0 = a.ctl[CTL_NOUT];
    int tok = a.ctl[CTL_TOK];
    // Norm weights (and q/k/v biases) go through shared memory in cp.async
    // groups, one per layer and one for the final norm, alternating between two
    // buffers: group g+1 is issued when group g's layer starts, so every norm
    // finds its weights copied during the previous layer.
    float *const bias0 = v.bias;
    auto issue_norms = [&](int grp) {
        const int st = grp / (L + 1), l = grp - st * (L + 1);
        float *nb = v.nw + (grp & 1) * 2 * a.dim;
        if (st < a.n_steps) {
            if (l < L) {
                const PLayer *Lp = p_layers + l;
                for (int i = tid; i < a.dim / 4; i += PT) {
                    cp_async16(nb + 4 * i, Lp->attn_norm + 4 * i);
                    cp_async16(nb + a.dim + 4 * i, Lp->ffn_norm + 4 * i);
                }
                if (a.has_bias)
                    for (int r = v.qkv0 + tid; r < qkv1; r += PT) {
                        const float *b = r < qd ? Lp->bq + r
                                                : (r < qd + a.nkv * a.hd ? Lp->bk + (r - qd)
                                                                         : Lp->bv + (r - qd - a.nkv * a.hd));
                        cp_async4(bias0 + (grp & 1) * 64 + (r - v.qkv0), b);
                    }
            } else {
                for (int i = tid; i < a.dim / 4; i += PT) cp_async16(nb + 4 * i, a.final_norm + 4 * i);
            }
        }
        cp_async_commit();
    };
    if (tid == 0) {
        build_pieces(a, t, gi, G);
        for (int s = 0; s < P_NSLOT; s++) {
            mbar_init(&g.full[s], 1);
            mbar_init(&g.empty[s], PNW);
        }
        fence_mbar_init();
    }
    __syncthreads();   // all 544 threads: the piece table and barriers are ready
    if (tid >= PT) {   // the producer warp
        if (tid == PT) ring_producer(a, t, g, v.ring);
        return true;
    }
    issue_norms(0);
    unsigned kc = 0;   // pieces consumed
    bool ok = true;
    const int role = gi == 0 ? 0 : (gi == G - 1 ? 1 : -1);
    (void)role;
    for (int step = 0; step < a.n_steps && ok; step++) {
        const uint32_t T = step_tag(T0, step, L);
        const bool probe_on = step == (a.n_steps > 1 ? 1 : 0);
        (void)probe_on;
        embed_row(a, tok, v.xf);
        for (int l = 0; l < L && ok; l++) {
            const uint32_t TL = T + 8u * (uint32_t)l;
            // the next layer's norm weights (and biases) start moving now
            const int grp = step * (L + 1) + l;
            issue_norms(grp + 1);
            const float *nw = v.nw + (grp & 1) * 2 * a.dim;
            v.bias = bias0 + (grp & 1) * 64;
            PPROBE(role, l, 0);
            if (l > 0) ok = gather_x(a, v.xf, a.w_x + a.dim, TL - 8u + TG_XB);
            if (!ok) break;
            PPROBE(role, l, 1);
#ifdef EMBER_PROBES
            if (tid == 0) p_detail = probe_on && role == 0 && l == 1;
            csync();
#endif
            for (int r = v.own0 + tid; r < v.own1; r += PT) v.xown[r - v.own0] = v.xf[r];
            norm_quant(a, v.xf, v.sq, v.xq, v.xd, nw);
            PPROBE(role, l, 2);
            ok = gemv_stage<PS_QKV>(a, t, g, v, l, TL + TG_QKV, kc);
            PPROBE(role, l, 3);
#ifdef EMBER_PROBES
            if (tid == 0) p_detail = 0;
#endif
            ok = ok && gather_q8(a, v.xq, v.xd, a.w_o, qd, TL + TG_O);
            PPROBE(role, l, 4);
            ok = ok && gemv_stage<PS_WO>(a, t, g, v, l, TL + TG_XA, kc);
            PPROBE(role, l, 5);
            ok = ok && gather_x(a, v.xf, a.w_x, TL + TG_XA);
            PPROBE(role, l, 6);
            if (!ok) break;
            norm_quant(a, v.xf, v.sq, v.xq, v.xd, nw + a.dim);
            PPROBE(role, l, 7);
            ok = gemv_stage<PS_W13>(a, t, g, v, l, TL + TG_H, kc);
            PPROBE(role, l, 8);
            ok = ok && gather_q8(a, v.xq, v.xd, a.w_h, a.hidden, TL + TG_H);
            PPROBE(role, l, 9);
            ok = ok && gemv_stage<PS_W2>(a, t, g, v, l, TL + TG_XB, kc);
            PPROBE(role, l, 10);
        }
        if (!ok) break;
        // final norm + lm_head, this CTA's argmax partial
        const uint32_t TH = T + 8u * (uint32_t)L;
        const int grp = step * (L + 1) + L;
        issue_norms(grp + 1);
        PPROBE(role, L, 0);
        if (!gather_x(a, v.xf, a.w_x + a.dim, TH - 8u + TG_XB)) { ok = false; break; }
        PPROBE(role, L, 1);
        norm_quant(a, v.xf, v.sq, v.xq, v.xd, v.nw + (grp & 1) * 2 * a.dim);
        if (tid == 0) { g.bv = -INFINITY; g.bi = 0x7FFFFFFF; g.nan0 = 0; }
        csync();
        PPROBE(role, L, 2);
        if (!gemv_stage<PS_HEAD>(a, t, g, v, 0, 0, kc)) { ok = false; break; }
        PPROBE(role, L, 3);
        if (step + 1 == a.n_steps && a.out_tokens == nullptr) break;   // forward: no pick
        if (tid == 0) {
            tw_store(a.w_am + 2 * gi, __float_as_uint(g.bv), TH);
            tw_store(a.w_am + 2 * gi + 1, g.nan0 ? 0xFFFFFFFFu : (uint32_t)g.bi, TH);
        }
        // the pick: first index of the maximum over every CTA's partial; a NaN
        // logit 0 keeps index 0 (ref src/sample.c:114-118)
        {
            uint32_t w[1];
            if (!tw_wait<1>(w, a.w_am, 2 * G, TH, a)) { ok = false; break; }
            float *pv = v.P;
            if (tid < 2 * G) pv[tid] = __uint_as_float(w[0]);
            csync();
            if (tid < 32) {
                float bv = -INFINITY;
                int bi = 0x7FFFFFFF, nan0 = 0;
                for (int c = tid; c < G; c += 32) {
                    const int ci = (int)__float_as_uint(pv[2 * c + 1]);
                    if (ci == -1) nan0 = 1;
                    else if (am_better(pv[2 * c], ci, bv, bi)) { bv = pv[2 * c]; bi = ci; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    nan0 |= __shfl_xor_sync(0xffffffffu, nan0, o);
                    if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (tid == 0) g.tok = (nan0 || bi == 0x7FFFFFFF) ? 0 : bi;
            }
            csync();
            tok = g.tok;
            if (gi == 0 && tid == 0 && a.out_tokens) a.out_tokens[nout0 + step] = tok;
            PPROBE(role, L, 4);
        }
    }
    if (!ok) {
        cp_async_wait_all();   // (the producer waits for the weight copies it issued)
        return false;
    }
    cp_async_wait_all();
    if (gi == 0 && tid == 0) {
        a.ctl[CTL_TOK] = tok;
        a.ctl[CTL_POS] = pos0 + a.n_steps;
        if (a.out_tokens) a.ctl[CTL_NOUT] = nout0 + a.n_steps;
        a.ctl[CTL_TAG] = (int)step_tag(T0, a.n_steps, L);
    }
    return true;
}

template <typename T>
EMB_DEV bool attn_cta(const PArgs &a, unsigned char *smem, const double *tab) {
    __shared__ __align__(16) AShared sh;
    const int tid = threadIdx.x, L = a.L;
    if (tid >= PT) return true;   // attention needs no producer warp
    const uint32_t T0 = (uint32_t)a.ctl[CTL_TAG];
    const int pos0 = a.ctl[CTL_POS];
    if (tid == 0) {
        mbar_init(&sh.vbar[0], 1);
        mbar_init(&sh.vbar[1], 1);
        fence_mbar_init();
        sh.vph[0] = sh.vph[1] = 0;
        sh.pending[0] = sh.pending[1] = 0;
    }
    csync();
    attn_prefetch<T>(a, sh, smem, 0, pos0);
    bool ok = true;
    const int role = blockIdx.x == 0 ? 2 : ((int)blockIdx.x == a.n_att - 1 ? 3 : -1);
    for (int step = 0; step < a.n_steps && ok; step++) {
        const int pos = pos0 + step;
        const uint32_t TS = step_tag(T0, step, L);
        const bool probe_on = step == (a.n_steps > 1 ? 1 : 0);
        for (int l = 0; l < L && ok; l++) {
            const uint32_t TL = TS + 8u * (uint32_t)l;
            ok = attn_stage<T>(a, sh, smem, tab, l, pos, TL + TG_QKV, TL + TG_O, role, probe_on);
            if (!ok) break;
            // the next layer's cache (or, after the last layer, the next step's
            // first layer, which includes this step's position)
            if (l + 1 < L) attn_prefetch<T>(a, sh, smem, l + 1, pos);
            else if (step + 1 < a.n_steps) attn_prefetch<T>(a, sh, smem, 0, pos + 1);
        }
    }
    if (!ok) {
        cp_async_wait_all();
        if (tid == 0)
            for (int i = 0; i < 2; i++)
                if (sh.pending[i])
                    for (uint32_t k = 0; k < MBAR_TRIES; k++)
                        if (mbar_try_wait(&sh.vbar[i], sh.vph[i])) break;
        csync();
    }
    return ok;
}

// One launch: n_steps token steps (greedy picks between them when out_tokens is
// set; a single forward step otherwise). Cooperative launch: every CTA resident.
template <typename T>
__global__ void __launch_bounds__(PTT, 1) ember_persist_kernel(const __grid_constant__ PArgs a) {
    unsigned char *const smem = p_dyn;
    __shared__ double tab[64];
    expf_table_load(tab, a.ex);
    for (int i = threadIdx.x; i < a.L * (int)(sizeof(PLayer) / 8); i += PTT)
        reinterpret_cast<unsigned long long *>(p_layers)[i] = reinterpret_cast<const unsigned long long *>(a.layers)[i];
    __syncthreads();
    if ((int)blockIdx.x < a.n_att) attn_cta<T>(a, smem, tab);
    else gemv_cta(a, smem, tab, (int)blockIdx.x - a.n_att, (int)gridDim.x - a.n_att);
}

}  // namespace emb
