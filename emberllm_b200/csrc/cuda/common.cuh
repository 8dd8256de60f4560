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

// Bytes of one quantized row: Q8_0 32 int8 per block, Q4_0 16 bytes per block.
__host__ __device__ inline size_t qrow_bytes(int dtype, int cols) {
    return dtype == EMBER_DT_Q4_0 ? (size_t)cols / 2 : (dtype == EMBER_DT_Q8_0 ? (size_t)cols : (size_t)cols * 4);
}

// ---- programmatic dependent launch (PDL) -----------------------------------
// Every kernel of the token step is launched with programmatic stream
// serialization: it lets the NEXT kernel start as soon as all of its CTAs have
// begun (launch_dependents), and waits for the PREVIOUS kernel to finish and
// flush its memory (wait) before touching anything that kernel wrote. The span
// between the two is used to prefetch this kernel's weights into L2.
EMB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
EMB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Bulk L2 prefetch of [p, p+bytes); p 16-byte aligned, bytes a multiple of 16.
EMB_DEV void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The device expf: the host C library's expf, reproduced from the recipe and
// exception table described in expf_core.h.
struct ExpfDev {
    EmberExpfParams p;      // p.slots is a DEVICE pointer here
};

EMB_DEV float expf_exact(const ExpfDev &e, float x) { return exc_expf(&e.p, e.p.slots, x); }

}  // namespace emb
