// head.cuh — the last kernel of a token step: final RMSNorm, the lm_head GEMV
// over the vocabulary and, for device greedy decoding, the argmax with the
// token / position advance (ref src/model.c:411-412, src/sample.c:114-118).
//
// The lm_head matrix is the step's largest read (vocab x dim Q8_0: 166 MB for
// Qwen3-0.6B) and its arithmetic is small, so the kernel is a stream. One CTA
// per SM owns a contiguous range of 32-row groups:
//   - a producer warp (one lane) moves each group -- its 32 quantized rows and
//     their fp16 scales, two contiguous ranges -- into a ring of shared-memory
//     stages with bulk asynchronous copies completing on "full" mbarriers; the
//     first stages are issued before the programmatic-launch wait, so they
//     overlap the previous kernel and the RMSNorm prologue (the ring's depth,
//     not the arithmetic, sets the kernel's bandwidth: measured 58 / 42 / 36 /
//     33 / 32 us for 2..6 stages of 34 KB on Qwen3-0.6B; an L2 prefetch of each
//     stage's next group did not help);
//   - consumer warp w (one per stage, up to 8) takes the groups of stage w,
//     w, w+S, w+2S, ... in order. Lane b holds block b of the quantized
//     activation in registers and forms, for each row, the block term
//     ((float)dot * d_w) * d_x; the terms go back into the stage's row space
//     (transposed, stride 33), lane r adds row r's terms in block order -- the
//     reference's sequential row sum (src/kernels.c:152-164) -- and the stage
//     is released ("empty" mbarrier) for the group S places later.
// Every mbarrier wait is bounded (common.cuh): a lost copy records an error in
// the device error word and the kernel returns.
//
// Greedy tail: each lane keeps the first index of the strict maximum over its
// rows; warps, then CTAs merge (the order-free rule "larger value, then smaller
// index"; NaN never wins) and the last CTA to finish (a ticket) writes the
// token, advances the position and appends the token to the output list, with
// the reference's rule that a NaN at index 0 keeps index 0.
#pragma once

#include "kernels.cuh"

namespace emb {

constexpr int HEAD_CW = 8;                          // consumer warps
constexpr int HEAD_THREADS = 32 * (HEAD_CW + 1);    // + the producer warp
constexpr int HEAD_MAX_STAGES = 8;
static_assert(HEAD_MAX_STAGES <= HEAD_CW, "one consumer warp per ring stage");
constexpr int HEAD_TS = 33;                         // transpose row stride (floats)
constexpr int HEAD_T_BYTES = 32 * HEAD_TS * 4;      // one warp's transpose buffer

struct HeadArgs {
    const uint8_t *q;       // lm_head rows, Q8_0 (32 B per block) or Q4_0 (16 B)
    const __half *s;        // fp16 scales [rows][cols/32]
    int rows, cols, groups; // vocab, dim, ceil(rows/32)
    int stages, stage_bytes;
    const float *x;         // the residual stream
    const float *norm_w;    // final norm weights
    float eps;
    float *logits;
    int *err;
    // greedy tail
    float *part_v;          // [gridDim.x]
    int *part_i;
    unsigned *ticket;       // zero between launches
    int *ctl;
    int *out;
};

// dynamic shared memory: the ring, the RMSNorm prologue's scratch (norm
// weights, x, squares), the quantized activation
__host__ inline size_t head_smem_bytes(int stages, int stage_bytes, int cols) {
    return (size_t)stages * stage_bytes + (size_t)cols * 12 + pad16(cols) + pad16((size_t)(cols / 32) * 4);
}

// a stage: 32 quantized rows (at least a transpose buffer's size: a consumer
// reuses the rows' space for its block terms) and 32 rows of scales
__host__ __device__ inline size_t head_q_bytes(int q4, int cols) {
    const size_t rb = q4 ? (size_t)cols / 2 : (size_t)cols;
    return 32 * rb > (size_t)HEAD_T_BYTES ? 32 * rb : (size_t)HEAD_T_BYTES;
}
__host__ __device__ inline int head_stage_bytes(int q4, int cols) {
    return (int)((head_q_bytes(q4, cols) + pad16((size_t)32 * (cols / 32) * 2) + 127) / 128 * 128);
}

// group g (rows 32g .. 32g+31) into stage `dst`, completing on `bar`. Row bytes
// and scale rows start on 16-byte boundaries (row bytes are multiples of 16;
// 32 rows of scales are 64*nb bytes); the scales are padded on the device, so
// rounding their size up to 16 bytes stays in bounds.
template <bool Q4>
EMB_DEV void head_issue(const HeadArgs &a, int g, unsigned char *dst, uint64_t *bar) {
    const size_t rb = Q4 ? (size_t)a.cols / 2 : (size_t)a.cols;
    const int nb = a.cols / 32, row0 = g * 32, nrows = min(32, a.rows - row0);
    const uint32_t qb = (uint32_t)(nrows * rb), sb = (uint32_t)pad16((size_t)nrows * nb * 2);
    mbar_expect_tx(bar, qb + sb);
    bulk_g2s(dst, a.q + (size_t)row0 * rb, qb, bar);
    bulk_g2s(dst + head_q_bytes(Q4, a.cols), a.s + (size_t)row0 * nb, sb, bar);
}

template <bool ARGMAX, bool Q4>
__global__ void __launch_bounds__(HEAD_THREADS, 1) lm_head_kernel(const HeadArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[HEAD_MAX_STAGES], empty[HEAD_MAX_STAGES];
    __shared__ float wv[HEAD_CW + 1];
    __shared__ int wi[HEAD_CW + 1];
    __shared__ bool last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cols = a.cols, nb = cols / 32, S = a.stages;
    const size_t rb = Q4 ? (size_t)cols / 2 : (size_t)cols;
    const int g0 = (int)((long long)blockIdx.x * a.groups / gridDim.x);
    const int ng = (int)((long long)(blockIdx.x + 1) * a.groups / gridDim.x) - g0;
    unsigned char *ring = smem;
    float *nw_s = reinterpret_cast<float *>(smem + (size_t)S * a.stage_bytes);
    float *x_s = nw_s + cols, *sq_s = nw_s + 2 * cols;
    int8_t *xq_s = reinterpret_cast<int8_t *>(nw_s + 3 * cols);
    float *xd_s = reinterpret_cast<float *>(xq_s + pad16(cols));
    constexpr int PW = HEAD_CW;   // the producer warp

    // ---- pre-wait: weights only ----
    if (tid == PW * 32) {
        for (int st = 0; st < S; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 1);
        }
        fence_mbar_init();
        for (int j = 0; j < S && j < ng; j++) head_issue<Q4>(a, g0 + j, ring + (size_t)j * a.stage_bytes, &full[j]);
    }
    for (int i = tid; i < cols; i += HEAD_THREADS) nw_s[i] = a.norm_w[i];
    pdl_wait_then_release();

    // ---- RMSNorm (ref src/model.c:50-55) and the Q8_0 activation ----
    for (int i = tid; i < cols; i += HEAD_THREADS) {
        const float v = a.x[i];
        x_s[i] = v;
        sq_s[i] = fmul(v, v);
    }
    __syncthreads();
    const float sc = rms_scale(split_chain_sum<HEAD_THREADS>(sq_s, cols), cols, a.eps);
    // normalize (x*scale)*w and quantize (ref src/kernels.c:211): eight threads per
    // 32-block, four elements each, each thread normalizing the four it quantizes
    for (int base = 0; base < nb * 8; base += HEAD_THREADS) {
        const int q8 = base + tid;
        const bool act = q8 < nb * 8;
        const unsigned mask = __ballot_sync(0xffffffffu, act);
        if (act) {
            const int b = q8 >> 3, sub = q8 & 7;
            float4 v = reinterpret_cast<const float4 *>(x_s + b * 32)[sub];
            const float4 w = reinterpret_cast<const float4 *>(nw_s + b * 32)[sub];
            v.x = fmul(fmul(v.x, sc), w.x);
            v.y = fmul(fmul(v.y, sc), w.y);
            v.z = fmul(fmul(v.z, sc), w.z);
            v.w = fmul(fmul(v.w, sc), w.w);
            float dq;
            const uint32_t packed = quant_quad(v, mask, &dq);
            reinterpret_cast<uint32_t *>(xq_s + b * 32)[sub] = packed;
            if (sub == 0) xd_s[b] = dq;
        }
    }
    __syncthreads();

    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    if (warp == PW) {
        if (lane == 0) {
            for (int j = S; j < ng; j++) {
                const int st = j % S;
                mbar_wait(&empty[st], (uint32_t)((j / S - 1) & 1), a.err, ERR_GEMV_WAIT);
                head_issue<Q4>(a, g0 + j, ring + (size_t)st * a.stage_bytes, &full[st]);
            }
            // every copy of this CTA has landed before it exits (the consumers
            // waited for them; a wait that gave up leaves this bounded drain)
            for (int st = 0; st < S && st < ng; st++)
                mbar_wait(&full[st], (uint32_t)(((ng - 1 - st) / S) & 1), a.err, ERR_GEMV_WAIT);
        }
    } else {
        // lane b: block b of the activation. For Q8_0 the two 16-byte halves of
        // a weight block are read in a lane-dependent order, so the eight lanes
        // of one shared-memory phase hit eight distinct bank groups; the
        // activation halves are paired accordingly (an integer dot is exact in
        // any order).
        const int c0 = Q4 ? 0 : (lane >> 2) & 1;
        int4 xa = make_int4(0, 0, 0, 0), xb = xa;
        float dx = 0.0f;
        int sx = 0;
        if (lane < nb) {
            const int4 *xp = reinterpret_cast<const int4 *>(xq_s + lane * 32);
            xa = xp[c0];
            xb = xp[c0 ^ 1];
            dx = xd_s[lane];
            if (Q4) {
                const int ones = 0x01010101;
                sx = __dp4a(xa.x, ones, sx); sx = __dp4a(xa.y, ones, sx); sx = __dp4a(xa.z, ones, sx);
                sx = __dp4a(xa.w, ones, sx); sx = __dp4a(xb.x, ones, sx); sx = __dp4a(xb.y, ones, sx);
                sx = __dp4a(xb.z, ones, sx); sx = __dp4a(xb.w, ones, sx);
            }
        }
        // warp w < S owns stage w and its groups w, w+S, w+2S, ...: the uses of
        // a stage are waited for in order by one warp, so each parity wait is
        // for the barrier's current phase (a waiter two phases ahead would pass
        // at once)
        const int st = warp;
        unsigned char *sq = ring + (size_t)st * a.stage_bytes;
        const __half *ss = reinterpret_cast<const __half *>(sq + head_q_bytes(Q4, cols));
        float *Tw = reinterpret_cast<float *>(sq);   // block terms, once the rows are read
        for (int j = warp; warp < S && j < ng; j += S) {
            mbar_wait(&full[st], (uint32_t)((j / S) & 1), a.err, ERR_GEMV_WAIT);
            const int row0 = (g0 + j) * 32, nrows = min(32, a.rows - row0);
            float t[32];
#pragma unroll
            for (int r = 0; r < 32; r++) {
                t[r] = 0.0f;
                if (lane < nb && r < nrows) {
                    int acc;
                    if (Q4) {
                        // Q4_0: element i is nibble (byte i & 15) - 8, element
                        // i+16 is (byte i >> 4) - 8 (ref src/kernels.c:175-179)
                        const uint4 v = *reinterpret_cast<const uint4 *>(sq + r * rb + lane * 16);
                        const uint32_t m = 0x0F0F0F0Fu;
                        const int4 lo = make_int4((int)(v.x & m), (int)(v.y & m), (int)(v.z & m), (int)(v.w & m));
                        const int4 hi = make_int4((int)((v.x >> 4) & m), (int)((v.y >> 4) & m),
                                                  (int)((v.z >> 4) & m), (int)((v.w >> 4) & m));
                        acc = dp8(lo, hi, xa, xb) - 8 * sx;
                    } else {
                        const int4 *wp = reinterpret_cast<const int4 *>(sq + r * rb + lane * 32);
                        acc = dp8(wp[c0], wp[c0 ^ 1], xa, xb);
                    }
                    t[r] = fmul(fmul(__int2float_rn(acc), __half2float(ss[r * nb + lane])), dx);
                }
            }
            __syncwarp();   // every lane has read the rows: their space takes the terms
            if (lane < nb) {
#pragma unroll
                for (int r = 0; r < 32; r++) Tw[r * HEAD_TS + lane] = t[r];
            }
            __syncwarp();
            float s = 0.0f;
            if (lane < nrows) s = chain_sum(0.0f, Tw + lane * HEAD_TS, nb);
            // generic writes to the stage precede the next bulk copy into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);   // the stage is free for group j + S
            if (lane < nrows) {
                a.logits[row0 + lane] = s;
                if (ARGMAX) am_merge(bv, bi, s, row0 + lane);
            }
        }
    }
    // ---- greedy tail (ref src/sample.c:114-118) ----
    if constexpr (ARGMAX) {
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i = __shfl_xor_sync(0xffffffffu, bi, o);
            am_merge(bv, bi, v, i);
        }
        __threadfence();   // this thread's logits before the ticket
        if (lane == 0) {
            wv[warp] = bv;
            wi[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float v = wv[0];
            int i = wi[0];
            for (int w = 1; w <= HEAD_CW; w++) am_merge(v, i, wv[w], wi[w]);
            a.part_v[blockIdx.x] = v;
            a.part_i[blockIdx.x] = i;
            __threadfence();
            last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (last && tid == 0) {
            __threadfence();
            float v = -INFINITY;
            int idx = 0x7FFFFFFF;
            for (int b = 0; b < (int)gridDim.x; b++)
                am_merge(v, idx, *(volatile float *)&a.part_v[b], *(volatile int *)&a.part_i[b]);
            if (idx == 0x7FFFFFFF || isnan(*(volatile float *)&a.logits[0])) idx = 0;
            a.ctl[CTL_TOK] = idx;
            a.ctl[CTL_POS] += 1;
            if (a.out) a.out[a.ctl[CTL_NOUT]] = idx;
            a.ctl[CTL_NOUT] += 1;
            *a.ticket = 0;
        }
    }
}

}  // namespace emb
