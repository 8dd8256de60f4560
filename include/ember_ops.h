/* ember_ops.h — op-level and runtime entry points that emberllm exports from its
 * library besides the public API (its src/kernels.h and src/util.h).
 *
 * emberllm's CLI and server call the thread-pool functions, and its shared
 * library exports the quantizers, fp16 helpers and matmuls; this library keeps
 * every one of those symbols with the same signature so that a caller linked
 * against emberllm's libember links against libember_b200 unchanged:
 *
 *   - ember_matmul / ember_matmul_batch run on the GPU (host pointers in and out,
 *     copies inside). They are the op-level parity entry points: same inputs,
 *     bit-identical outputs to the reference's CPU kernels, including the
 *     quantized activation written to `xq`.
 *   - ember_quantize_q8_0 / _q4_0 and the fp16 helpers are host functions: they
 *     serve the offline requantizer (ember_quantize_file), not the token loop,
 *     whose activation quantization happens inside the GPU kernels.
 *   - the thread-pool functions are kept as callable no-ops; the CUDA grid
 *     replaces emberllm's pthread pool.
 */
#ifndef EMBER_B200_OPS_H
#define EMBER_B200_OPS_H

#include "ember.h"

#ifdef __cplusplus
extern "C" {
#endif

#pragma pack(push, 1)
/* quant blocks exactly as stored in .ember files (ref src/kernels.h:46-51) */
typedef struct { uint16_t d; int8_t  qs[EMBER_Q_BLOCK];     } BlockQ8_0;  /* 34 B */
typedef struct { uint16_t d; uint8_t qs[EMBER_Q_BLOCK / 2]; } BlockQ4_0;  /* 18 B */
#pragma pack(pop)

/* IEEE binary16 <-> binary32, round-to-nearest-even (ref src/kernels.c:25-68) */
float    ember_f16_to_f32(uint16_t h);
uint16_t ember_f32_to_f16(float f);

/* per-32-block symmetric quantizers (ref src/kernels.c:73-115); n % 32 == 0 */
void ember_quantize_q8_0(const float *x, BlockQ8_0 *out, int n);
void ember_quantize_q4_0(const float *x, BlockQ4_0 *out, int n);

/* out[d_out] = W[d_out, n_in] x[n_in] on the GPU (replaces ref src/kernels.c:207-220).
 * For quantized W the activation is quantized to Q8_0 into xq (n_in/32 blocks,
 * host memory, filled on return) exactly as the reference does. */
void ember_matmul(float *out, const float *x, const void *w, int dtype,
                  int n_in, int d_out, BlockQ8_0 *xq);
/* out[B][d_out] = x[B][n_in] W^T on the GPU (replaces ref src/kernels.c:250-264);
 * xq receives B*(n_in/32) blocks for quantized W. */
void ember_matmul_batch(float *out, const float *x, const void *w, int dtype,
                        int n_in, int d_out, int B, BlockQ8_0 *xq);

/* emberllm's pthread pool API (ref src/kernels.h:75-85). No-ops that remember the
 * requested count, so `--threads N` and the server keep working. */
typedef void (*EmberRangeFn)(void *ctx, int i0, int i1);
void ember_threads_init(int nthreads);
void ember_threads_shutdown(void);
int  ember_nthreads(void);
void ember_parallel_for(EmberRangeFn fn, void *ctx, int n);
int  ember_should_parallel(long work);

/* fatal-error convention (ref src/util.c:8-34): "ember: <msg>" on stderr, exit(1);
 * the allocators never return NULL. */
void  ember_die(const char *fmt, ...);
void *ember_xmalloc(size_t n, const char *what);
void *ember_xcalloc(size_t count, size_t size, const char *what);
void *ember_xrealloc(void *p, size_t n, const char *what);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* EMBER_B200_OPS_H */
