// common.cuh — device helpers shared by the token-loop kernels.
//
// Exactness rules. The reference's deterministic build evaluates every fp32
// expression as written, one IEEE operation at a time, with no fused
// multiply-add (-ffp-contract=off) and no reassociation. Its int8 re-quantization
// of each activation makes the logits sensitive to single-ulp differences, so
// the kernels here spell every floating-point step that feeds a quantization,
// the KV cache or the logits with the round-to-nearest intrinsics below (which
// the compiler never contracts), in the reference's order. Integer block dot
// products are exact in any order and use dp4a freely. The library is also
// compiled with --fmad=false as a second line of defence.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ember_cuda.h"
#include "expf_core.h"

#define EMB_DEV static __device__ __forceinline__

namespace emb {

EMB_DEV float fadd(float a, float b) { return __fadd_rn(a, b); }
EMB_DEV float fsub(float a, float b) { return __fsub_rn(a, b); }
EMB_DEV float fmul(float a, float b) { return __fmul_rn(a, b); }
EMB_DEV float fdiv(float a, float b) { return __fdiv_rn(a, b); }
EMB_DEV float fsqrt(float a) { return __fsqrt_rn(a); }

// lroundf: nearest integer, halfway cases away from zero. |v| < 2^23 here, so
// v - trunc(v) is exact.
EMB_DEV float round_half_away(float v) {
    float t = truncf(v);
    float frac = fabsf(__fsub_rn(v, t));
    return frac >= 0.5f ? __fadd_rn(t, copysignf(1.0f, v)) : t;
}

// RMSNorm scale as the reference computes it after its sequential sum of
// squares: 1.0f / sqrtf(ss / n + eps) (ref src/model.c:53).
EMB_DEV float rms_scale(float ss, int n, float eps) {
    return fdiv(1.0f, fsqrt(fadd(fdiv(ss, (float)n), eps)));
}

EMB_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Quantize one 32-element block held one element per lane (ref
// src/kernels.c:73-92): d = amax/127 in fp32, id = 1/d (from the unrounded d),
// q = lroundf(x*id) clamped to +-127; the scale used downstream is d rounded to
// fp16 and widened back (ref src/kernels.c:84 and :163). Returns q; *dq gets the
// widened scale. The max of |x| is order-free.
EMB_DEV int8_t quant_lane(float x, float *dq) {
    float amax = warp_max(fabsf(x));
    float d = fdiv(amax, 127.0f);
    float id = d > 0.0f ? fdiv(1.0f, d) : 0.0f;
    *dq = __half2float(__float2half_rn(d));
    float q = round_half_away(fmul(x, id));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return (int8_t)(int)q;
}

// Quantize four consecutive elements of a 32-block whose eight quads sit in
// eight consecutive lanes (lanes of one block all active, in `mask`): the same
// arithmetic as quant_lane, the block max reduced over the eight lanes. Returns
// the four int8 codes packed little-endian.
EMB_DEV uint32_t quant_quad(float4 v, unsigned mask, float *dq) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 4));
    const float d = fdiv(amax, 127.0f);
    const float id = d > 0.0f ? fdiv(1.0f, d) : 0.0f;
    *dq = __half2float(__float2half_rn(d));
    float q[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float t = fminf(fmaxf(round_half_away(fmul(q[j], id)), -127.0f), 127.0f);
        packed |= (uint32_t)(uint8_t)(int8_t)(int)t << (8 * j);
    }
    return packed;
}

// int8 dot of one Q8_0 weight block (32 B) with one activation block, both in smem
EMB_DEV int dot_q8_block(const uint8_t *w, const int8_t *xq) {
    int4 w0 = reinterpret_cast<const int4 *>(w)[0];
    int4 w1 = reinterpret_cast<const int4 *>(w)[1];
    int4 a0 = reinterpret_cast<const int4 *>(xq)[0];
    int4 a1 = reinterpret_cast<const int4 *>(xq)[1];
    int acc = 0;
    acc = __dp4a(w0.x, a0.x, acc); acc = __dp4a(w0.y, a0.y, acc);
    acc = __dp4a(w0.z, a0.z, acc); acc = __dp4a(w0.w, a0.w, acc);
    acc = __dp4a(w1.x, a1.x, acc); acc = __dp4a(w1.y, a1.y, acc);
    acc = __dp4a(w1.z, a1.z, acc); acc = __dp4a(w1.w, a1.w, acc);
    return acc;
}

// int8 dot of 32 weight bytes (two int4) with 32 activation bytes, exact in int32
EMB_DEV int dp8(int4 w0, int4 w1, int4 a0, int4 a1) {
    int acc = 0;
    acc = __dp4a(w0.x, a0.x, acc); acc = __dp4a(w0.y, a0.y, acc);
    acc = __dp4a(w0.z, a0.z, acc); acc = __dp4a(w0.w, a0.w, acc);
    acc = __dp4a(w1.x, a1.x, acc); acc = __dp4a(w1.y, a1.y, acc);
    acc = __dp4a(w1.z, a1.z, acc); acc = __dp4a(w1.w, a1.w, acc);
    return acc;
}

// Q4_0 block (16 B): element i is nibble (byte i & 15) - 8, element i+16 is
// (byte i >> 4) - 8 (ref src/kernels.c:175-179). Unsigned nibbles fit in a
// signed byte, so sum((n-8)*a) = sum(n*a) - 8*sum(a), all exact in int32.
EMB_DEV int dot_q4_block(const uint8_t *w, const int8_t *xq) {
    uint4 v = reinterpret_cast<const uint4 *>(w)[0];
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

// Bytes of one row in the device layout: Q8_0 32 int8 per block, Q4_0 16 bytes
// per block, fp32 4 bytes per element.
__host__ __device__ inline size_t qrow_bytes(int dtype, int cols) {
    return dtype == EMBER_DT_Q4_0 ? (size_t)cols / 2 : (dtype == EMBER_DT_Q8_0 ? (size_t)cols : (size_t)cols * 4);
}

// ---- programmatic dependent launch (PDL) -----------------------------------
// Every kernel of the token step is launched with programmatic stream
// serialization and begins with
//
//     [pre-wait work]  griddepcontrol.wait  griddepcontrol.launch_dependents ...
//
// The wait returns when the previous kernel (N-1) has finished and flushed its
// memory; only then does this kernel (N) allow the next one (N+1) to launch.
// Consequently, when kernel N+1 starts its pre-wait work, every CTA of kernel N
// has passed its wait, so kernel N-1 and everything before it is complete: the
// pre-wait work of a kernel may read weights, tables, and anything written two
// or more launches earlier (the KV cache of previous positions, the step's
// position word), and must not read what its immediate predecessor writes.
// 16-byte global -> shared copies that complete asynchronously (cp.async):
// issue, commit the group, and wait for all groups before reading the data
EMB_DEV void cp_async16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
EMB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
EMB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// wait until at most one committed group (the newest) is still in flight
EMB_DEV void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

EMB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
EMB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- optional phase probes ----------------------------------------------------
// Built only with -DEMBER_PROBES (a separate profiling build): CTA 0 records the
// global timer at named phase boundaries of each kernel kind (the last launch of
// each kind wins), and every launch records when it reached and left its
// dependency wait. They record timestamps only and change no computation.
#ifdef EMBER_PROBES
__device__ unsigned long long g_probe[8][16];
__device__ unsigned g_wait_count;
__device__ unsigned long long g_wait_times[8192][2];
EMB_DEV unsigned long long probe_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define EMB_PROBE(kind, slot)                                                     \
    do {                                                                          \
        if (blockIdx.x == 0 && threadIdx.x == 0) g_probe[kind][slot] = probe_now(); \
    } while (0)
EMB_DEV void pdl_wait_then_release() {
    unsigned long long t0 = probe_now();
    pdl_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned id = atomicAdd(&g_wait_count, 1u) & 8191u;
        g_wait_times[id][0] = t0;
        g_wait_times[id][1] = probe_now();
    }
    pdl_launch_dependents();
}
#else
#define EMB_PROBE(kind, slot) \
    do {                      \
    } while (0)
EMB_DEV void pdl_wait_then_release() {
    pdl_wait();
    pdl_launch_dependents();
}
#endif

// ---- exact sequential sums ---------------------------------------------------
// sum = ((0 + v[0]) + v[1]) + ... in index order: the reference's loop. The
// additions form one dependent chain; the loads are batched into registers
// ahead of it so the chain runs at the adder's latency.
EMB_DEV float chain_sum(float s, const float *v, int n) {
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        float r[16];
#pragma unroll
        for (int j = 0; j < 16; j++) r[j] = v[i + j];
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fadd_rn(s, r[j]);
    }
    for (; i < n; i++) s = __fadd_rn(s, v[i]);
    return s;
}

// chain_sum for long arrays: the next 16 loads are in flight while the current
// 16 values are added, so the chain runs at the adder's latency
EMB_DEV float chain_sum_pipe(float s, const float *v, int n) {
    if (n < 32) return chain_sum(s, v, n);
    float a[16], b[16];
#pragma unroll
    for (int j = 0; j < 16; j++) a[j] = v[j];
    int i = 16;
    for (; i + 32 <= n; i += 32) {
#pragma unroll
        for (int j = 0; j < 16; j++) b[j] = v[i + j];
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fadd_rn(s, a[j]);
#pragma unroll
        for (int j = 0; j < 16; j++) a[j] = v[i + 16 + j];
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fadd_rn(s, b[j]);
    }
    // a holds v[i-16 .. i-1]
#pragma unroll
    for (int j = 0; j < 16; j++) s = __fadd_rn(s, a[j]);
    for (; i < n; i++) s = __fadd_rn(s, v[i]);
    return s;
}

// sum of v[i]*v[i] in index order (products rounded, then added); the squares
// of the next 16 elements are formed while the current 16 are added
EMB_DEV float chain_sumsq(const float *v, int n) {
    float s = 0.0f;
    int i = 0;
    if (n >= 32) {
        float a[16], b[16];
#pragma unroll
        for (int j = 0; j < 16; j++) a[j] = __fmul_rn(v[j], v[j]);
        i = 16;
        for (; i + 32 <= n; i += 32) {
#pragma unroll
            for (int j = 0; j < 16; j++) b[j] = __fmul_rn(v[i + j], v[i + j]);
#pragma unroll
            for (int j = 0; j < 16; j++) s = __fadd_rn(s, a[j]);
#pragma unroll
            for (int j = 0; j < 16; j++) a[j] = __fmul_rn(v[i + 16 + j], v[i + 16 + j]);
#pragma unroll
            for (int j = 0; j < 16; j++) s = __fadd_rn(s, b[j]);
        }
        // a holds the squares of v[i-16 .. i-1]
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fadd_rn(s, a[j]);
    }
    for (; i < n; i++) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    return s;
}

// ---- a sequential sum of non-negative terms in a fraction of the chain's latency ----
// sum = ((0 + v[0]) + v[1]) + ... + v[n-1] in index order, exactly as
// chain_sum(0, v, n), computed by the block's NT threads over K segments of
// m = n/K terms at once: one thread adds segment 0 from 0; for each later
// segment k, NC threads add it from the NC consecutive floats centred on a
// double estimate of the exact sum of the segments before it. The float sum of
// i non-negative terms lies within (i-1)/2 ulps of the exact one and in practice
// within a few (the roundings largely cancel). Walking the boundaries in order,
// the chain that started from the float sum actually reached is the next sum.
// When a boundary's sum falls outside its window (or is not finite) the rest is
// added sequentially from there: the result is the loop's either way, only the
// time differs. v: shared memory, 16-byte aligned; n a multiple of 16*K (else
// one thread adds). The code stays small on purpose: it runs once per launch
// from a cold instruction cache, where every extra instantiation costs time.
template <int NT, int K = 4>
EMB_DEV float split_chain_sum(const float *v, int n, int *hit = nullptr) {
    constexpr int NC = 64, NB = K - 1;
    static_assert(K >= 2 && NT >= NC * NB + 1 && NT % 32 == 0, "split_chain_sum: block too small");
    __shared__ double red[NB][NT / 32];
    __shared__ float cand[NB][NC];
    __shared__ float first_part, answer;
    const unsigned FULL = 0xffffffffu;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (n % (16 * K) != 0 || n < 32 * K) {
        __syncthreads();
        if (tid == 0) answer = chain_sum(0.0f, v, n);
        __syncthreads();
        if (hit) *hit = 0;
        return answer;
    }
    const int m = n / K;
    // exact sums of segments 0..K-2, estimated in double (same order in every thread)
    double d[NB];
#pragma unroll
    for (int k = 0; k < NB; k++) d[k] = 0.0;
    for (int i = tid; i < m; i += NT) {
#pragma unroll
        for (int k = 0; k < NB; k++) d[k] = __dadd_rn(d[k], (double)v[k * m + i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int k = 0; k < NB; k++) d[k] = __dadd_rn(d[k], __shfl_down_sync(FULL, d[k], o));
    }
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < NB; k++) red[k][warp] = d[k];
    }
    __syncthreads();
    // window starts b0[k] for the sum of segments 0..k (the start of segment k+1)
    uint32_t b0[NB];
    bool finite = true;
    double D = 0.0;
#pragma unroll
    for (int k = 0; k < NB; k++) {
#pragma unroll
        for (int w = 0; w < NT / 32; w++) D = __dadd_rn(D, red[k][w]);
        const uint32_t bc = __float_as_uint(__double2float_rn(D));
        finite = finite && bc < 0x7F000000u;
        b0[k] = bc > NC / 2 ? bc - NC / 2 : 0u;
    }
    if (tid <= NC * NB) {
        const bool is_first = tid == NC * NB;
        const int kk = is_first ? 0 : tid / NC, j = tid % NC;
        uint32_t mine = b0[0];
#pragma unroll
        for (int k = 1; k < NB; k++) mine = kk == k ? b0[k] : mine;
        float s = is_first ? 0.0f : __uint_as_float(mine + (uint32_t)j);
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
        if (is_first) first_part = s;
        else cand[kk][j] = s;
    }
    __syncthreads();
    // walk the boundaries: s = the float sum of segments 0..k
    float s = first_part;
    int done = 1;   // segments summed into s
#pragma unroll
    for (int k = 0; k < NB; k++) {
        const uint32_t jk = __float_as_uint(s) - b0[k];
        if (done == k + 1 && finite && jk < (uint32_t)NC) {
            s = cand[k][jk];
            done = k + 2;
        }
    }
    if (hit) *hit = done == K;
    if (done == K) return s;
    if (tid == 0) answer = chain_sum(s, v + done * m, n - done * m);
    __syncthreads();
    return answer;
}

// ---- bulk async copies (TMA, non-tensor form) and mbarriers ----------------
EMB_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

EMB_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// make mbarrier initialisation visible to the async (TMA) proxy
EMB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

EMB_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// global -> shared bulk copy completing on `bar`; dst, src 16-byte aligned,
// bytes a multiple of 16; the copy lands in this CTA only.
EMB_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

EMB_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

EMB_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: each try_wait blocks for a hardware-chosen slice; after
// MBAR_TRIES slices (seconds in total) the wait gives up, records `code` in the
// device error word and returns false, so a lost copy can never hang the GPU.
constexpr uint32_t MBAR_TRIES = 1u << 22;
EMB_DEV bool mbar_wait_n(uint64_t *bar, uint32_t parity, int *err, int code, uint32_t tries) {
    for (uint32_t i = 0; i < tries; i++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, code);
    return false;
}
EMB_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    return mbar_wait_n(bar, parity, err, code, MBAR_TRIES);
}

// Bounded wait that backs off between polls (__nanosleep), for a thread whose
// wait may be long while other warps of the CTA work out of shared memory:
// a tight try_wait loop competes with their shared-memory accesses.
EMB_DEV bool mbar_wait_backoff(uint64_t *bar, uint32_t parity, int *err, int code) {
    for (uint32_t i = 0; i < MBAR_TRIES; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(256);
    }
    if (err) atomicExch(err, code);
    return false;
}

// CTA-wide wait: one thread waits on the mbarrier (acquiring the copied bytes),
// then a CTA barrier releases the others, who see the bytes through it.
EMB_DEV void mbar_wait_cta(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (threadIdx.x == 0) mbar_wait(bar, parity, err, code);
    __syncthreads();
}

// Bulk L2 prefetch of [p, p+bytes); p 16-byte aligned, bytes a multiple of 16.
EMB_DEV void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// KV cache element access: the cache holds fp32 as is, or fp16 rounded to
// nearest even (ref src/model.c:43, ember_f16c); reads widen to fp32
EMB_DEV float widen(float v) { return v; }
EMB_DEV float widen(__half v) { return __half2float(v); }
EMB_DEV void kv_round(float v, float *out) { *out = v; }
EMB_DEV void kv_round(float v, __half *out) { *out = __float2half_rn(v); }

// ctl words in device memory, read by the step's kernels (so one captured graph
// serves every position): pos, token, number of greedy tokens written, position
// of ids[0] during a prefill, and the device error word.
enum { CTL_POS = 0, CTL_TOK = 1, CTL_NOUT = 2, CTL_BASE = 3, CTL_ERR = 4, CTL_WORDS = 8 };

// device error codes (written to the state's error word, read by the host)
enum { ERR_NONE = 0, ERR_GEMV_WAIT = 1, ERR_ATTN_WAIT = 2, ERR_PF_WAIT = 3 };

// The device expf: the host C library's expf, reproduced from the recipe and
// exception table described in expf_core.h.
struct ExpfDev {
    EmberExpfParams p;      // p.slots is a DEVICE pointer here
};

// With the 64-entry 2^(j/64) table copied to shared memory (tab_s, by
// expf_table_load), so each call costs no global-memory latency; the exception
// slots stay in global memory (rarely read).
EMB_DEV float expf_exact(const ExpfDev &e, const double *tab_s, float x) {
    return exc_expf_t(&e.p, tab_s, e.p.slots, x);
}
// threads 0..63 copy the table (static data: may run before the dependency wait);
// the caller synchronises before the first expf_exact
EMB_DEV void expf_table_load(double *tab_s, const ExpfDev &e) {
    if (threadIdx.x < 64) tab_s[threadIdx.x] = e.p.tab[threadIdx.x];
}

}  // namespace emb
