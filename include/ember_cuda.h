/* ember_cuda.h — the thin C-ABI shim between the C11 host code and the sm_100a
 * kernels, plus the library's extension entry points.
 *
 * None of these functions has a counterpart in emberllm (which has no GPU
 * path); they are what the host side of this library (io.c / model.c, the
 * replacements of emberllm's src/io.c and src/model.c) calls to run the token
 * loop on the device. Every function returns 0 on success or a nonzero status,
 * with a message available from ember_cuda_error(); the host converts failures
 * into ember_die("cuda: ...") to keep emberllm's fatal-error convention.
 *
 * Only plain C types cross this boundary: host pointers, sizes, opaque handles.
 */
#ifndef EMBER_B200_CUDA_H
#define EMBER_B200_CUDA_H

#include <stdint.h>
#include "ember.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct EmberCudaModel EmberCudaModel;
typedef struct EmberCudaState EmberCudaState;

/* One 2-D weight as it sits in the host mapping. */
typedef struct {
    const void *data;   /* host pointer into the .ember mapping                     */
    int32_t dtype;      /* EMBER_DT_F32 / Q8_0 / Q4_0                                */
    int32_t rows;       /* output rows (d_out)                                       */
    int32_t cols;       /* input length (n_in)                                       */
} EmberCudaMat;

/* Everything the device needs from a model, resolved by the host (the same
 * tensors emberllm's ember_state_new_ex resolves, ref src/model.c:144-159).
 * Per-layer arrays have n_layers entries; optional vectors are NULL. */
typedef struct {
    int32_t dim, hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab;
    float   norm_eps;
    int32_t qk_norm;
    int32_t rope_neox;                   /* 1: NEOX half-split pairs, 0: interleaved */
    EmberCudaMat tok_emb, lm_head;       /* lm_head.data == tok_emb.data when tied */
    const float *final_norm;
    const EmberCudaMat *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    const float *const *attn_norm, *const *ffn_norm;
    const float *const *q_norm, *const *k_norm;   /* used when qk_norm != 0      */
    const float *const *b_q, *const *b_k, *const *b_v;
} EmberCudaModelDesc;

/* Parameters of the device expf. The device computes exp(x) with a fixed
 * double-precision recipe -- k = nearest integer to x*64/ln2, r = x - k*ln2/64
 * (ln2/64 in two parts), exp(x) = 2^(k>>6) * 2^((k&63)/64) * P(r) with P the
 * degree-5 Taylor polynomial and 2^(j/64) from a 64-entry table -- and rounds to
 * float. All constants and the table come from the host, so host and device
 * compute identical bits. The host scans every float input in [lo, hi] once
 * against the C library's expf and lists, in an open-addressing table, the
 * inputs where the library's result differs; the device consults the table only
 * when the double result lies within `window` units of 2^-29 float ulp of a
 * rounding midpoint (every listed input does, by construction) or the result is
 * not a normal float. Below lo the result is +0, above hi it is +inf. */
typedef struct {
    double coef[6];         /* polynomial coefficients, coef[k] ~ 1/k!                */
    double inv_step;        /* 64 / ln2                                               */
    double step_hi, step_lo;/* ln2 / 64 split so that k * step_hi is exact            */
    double shifter;         /* 1.5 * 2^52: rounds to the nearest integer              */
    uint32_t window;        /* midpoint window, units of 2^-29 float ulp              */
    float  lo, hi;          /* scanned input range                                    */
    uint32_t n_slots;       /* power of two                                           */
    uint32_t n_entries;
    const double *tab;      /* 64 doubles, 2^(j/64)                                   */
    const uint32_t *slots;  /* 2*n_slots words: (x bits, expf bits); empty key = ~0u */
} EmberExpfParams;

/* The double-precision exp recipe shared by host and device (see above). */
#define EMBER_EXPF_EMPTY 0xFFFFFFFFu

/* ---- device + model ---- */
/* Uploads (and repacks) the weights to the current device. `expf_params` is
 * copied. The device is EMBER_CUDA_DEVICE (default 0). */
int  ember_cuda_model_upload(const EmberCudaModelDesc *desc, const EmberExpfParams *expf_params,
                             EmberCudaModel **out);
void ember_cuda_model_free(EmberCudaModel *m);
/* bytes of weights the device holds for this model (after repacking) */
uint64_t ember_cuda_model_bytes(const EmberCudaModel *m);

/* ---- state ---- */
/* rope_cs: host table [ctx][head_dim/2][2] of (cos, sin), computed by the host
 * with the reference's own float expressions (ref src/model.c:69-71). */
int  ember_cuda_state_new(EmberCudaModel *m, int ctx, int kv_fp16, const float *rope_cs,
                          EmberCudaState **out);
void ember_cuda_state_free(EmberCudaState *s);

/* one decode step; copies vocab logits to host_logits (pinned or pageable) */
int  ember_cuda_forward(EmberCudaState *s, int tok, int pos, float *host_logits);
/* n tokens at start..start+n-1; last token's logits to host_logits */
int  ember_cuda_prefill(EmberCudaState *s, const int *ids, int n, int start, float *host_logits);
/* n_steps greedy steps without host round trips: step i feeds token t_i at pos+i
 * (t_0 = tok) and t_{i+1} = first argmax of its logits; writes t_1..t_n to
 * host_tokens and the last step's logits to host_logits (if not NULL). */
int  ember_cuda_greedy(EmberCudaState *s, int tok, int pos, int n_steps, int *host_tokens,
                       float *host_logits);

/* Profiling: runs one complete greedy step (token `tok` at `pos`, every kernel
 * of the step, no graph, no programmatic overlap) with a CUDA event before each
 * launch, and writes each launch's device time in ms to ms_out[0..*n_out). */
int  ember_cuda_profile_step(EmberCudaState *s, int tok, int pos, float *ms_out, int cap, int *n_out);

/* Device timing on the state's stream: record event `slot` (0..7), and the time
 * in ms between two recorded slots (waits for the later one). */
int  ember_cuda_mark(EmberCudaState *s, int slot);
int  ember_cuda_elapsed_ms(EmberCudaState *s, int a, int b, float *ms);
/* Mean device time of one kernel kind (0 qkv, 1 attention, 2 wo, 3 w1/w3+SwiGLU,
 * 4 w2, 5 lm_head), launched `reps` times for every layer in turn outside any
 * graph, and its algorithmic bytes per launch. Leaves the state usable only for
 * further timing (activations and cache are overwritten). */
int  ember_cuda_time_kernel(EmberCudaState *s, int kind, int reps, float *ms_per_launch,
                            double *bytes_per_launch);

/* Greedy pick without allocating: the first index of the largest of n device
 * floats `logits`, written to the device int `out_index`, enqueued on `stream`
 * (a cudaStream_t; NULL is the default stream). No counterpart in the reference.
 * For callers that cannot let the library allocate device memory (a host that
 * owns the GPU's memory through its own pool, or a per-token path that must not
 * risk cudaMalloc's synchronisation): it takes only caller-owned buffers and
 * keeps its scratch in a fixed array inside the library (about 2 KB per device,
 * held until exit). n must be in [1, 67108864]; other sizes are rejected with
 * status 1 and a line on stderr (2: bad pointer -- logits and out_index must be
 * device memory of one device, and a non-NULL stream must belong to it; 3: CUDA
 * error). The pick follows the reference's loop exactly: a NaN never wins, and a
 * NaN at index 0 gives 0. The work runs on the logits' device; the caller's
 * current device is unchanged on return. The first call on a device looks the
 * array up and should come before any stream capture; calls that overlap on the
 * GPU share the array and race. */
int  ember_cuda_argmax_static(const float *logits, int n, int *out_index, void *stream);

/* ---- batched greedy decode of independent streams ----
 * No counterpart in the reference (which decodes one sequence per state); this
 * is the many-sequence workload: n_streams independent sequences, each with its
 * own KV cache of ctx positions, advanced together. Up to 8 streams, the batch
 * holds one single-stream state per stream and runs their greedy steps at once
 * on separate CUDA streams. Beyond that (or with EMBER_BATCH=gemm), every step
 * runs all streams' tokens through the layers as one batch (tensor-core GEMMs
 * over the streams), each at its own position, then the final norm, lm_head and
 * a per-stream greedy pick. Per stream the arithmetic is the single-sequence
 * step's, so each stream's tokens and logits equal those of its own
 * ember_forward run. Requires Q8_0/Q4_0 layer and lm_head weights; n_streams in
 * [1, 512]. ember_cuda_batch_stream returns the stream of the batch (of its first
 * state when the batch holds one per stream). */
typedef struct EmberCudaBatch EmberCudaBatch;
int  ember_cuda_batch_new(EmberCudaModel *m, int n_streams, int ctx, int kv_fp16, const float *rope_cs,
                          int max_steps, EmberCudaBatch **out);
void ember_cuda_batch_free(EmberCudaBatch *b);
/* prompt ids[0..n) of stream `stream` at positions 0..n-1 (batched prefill into
 * the stream's cache); the last token's logits to host_logits (vocab floats) */
int  ember_cuda_batch_prefill(EmberCudaBatch *b, int stream, const int *ids, int n, float *host_logits);
/* n_steps greedy steps of every stream: stream i feeds toks[i] at pos[i], then
 * its own greedy picks. host_tokens (may be NULL) gets [n_steps][n_streams]
 * tokens; host_logits (may be NULL) the last step's logits [n_streams][vocab]. */
int  ember_cuda_batch_greedy(EmberCudaBatch *b, const int *toks, const int *pos, int n_steps, int *host_tokens,
                             float *host_logits);
void *ember_cuda_batch_stream(EmberCudaBatch *b);                /* cudaStream_t */

/* ---- sampling on the device ----
 * The settings of the reference's sampler (EmberSampler, ref src/ember.h:141-155)
 * that decide a draw: temperature, top_p, top_k, min_p and the three penalties. */
typedef struct {
    float   temperature, top_p;
    int32_t top_k;
    float   min_p, repeat_penalty, presence_penalty, frequency_penalty;
} EmberSampleParams;

/* The reference's ember_sample (src/sample.c:120-175) over the state's last
 * logits, on the device: penalties over hist[0..hist_len) (the sampler's history
 * array and length, in array order as the reference scans it), then greedy
 * (temperature <= 0) or temperature, softmax, stable descending order, top_k,
 * min_p, top_p and the draw r = u * cutoff, with u the reference's rng_f32 draw
 * (computed by the caller; ember_sample_device does it). The token to
 * *out_token; the state's logits are left as they were. No counterpart in the
 * reference (which samples on the host). */
int  ember_cuda_sample(EmberCudaState *s, const EmberSampleParams *p, float u, const int *hist, int hist_len,
                       int *out_token);

/* the state's pinned host logits buffer (vocab floats), owned by the state */
float       *ember_cuda_state_host_logits(EmberCudaState *s);

/* introspection for tests and benchmarks */
void        *ember_cuda_state_stream(EmberCudaState *s);      /* cudaStream_t */
const float *ember_cuda_state_logits_dev(EmberCudaState *s);  /* device pointer */
int          ember_cuda_state_launches_per_step(const EmberCudaState *s);
/* kernels of one device greedy token (the step, the lm_head with its fused
 * argmax or a separate argmax); 0 until the state has run a greedy step */
int          ember_cuda_state_launches_per_token(const EmberCudaState *s);
/* 1 when the state's decode steps run as the persistent kernel (one cooperative
 * launch per forward step or greedy run); 0 when they run as captured graphs of
 * per-stage kernels, with *why (if not NULL) naming the reason */
int          ember_cuda_state_persistent(const EmberCudaState *s, const char **why);
const char  *ember_cuda_error(void);
/* 1 if this library was built with sm_100a device code and a device is usable */
int          ember_cuda_available(void);

/* ---- host helpers implemented in C (glibc-dependent tables) ---- */
/* Builds (or loads from the cache directory $EMBER_CACHE_DIR, default
 * ~/.cache/ember_b200) the expf exception table for THIS host's C library.
 * The returned params point at static storage valid for the process. */
int  ember_host_expf_params(EmberExpfParams *out);
/* the device recipe evaluated on the host (identical bits); for tests */
float ember_host_expf_emulated(const EmberExpfParams *p, float x);
/* fills [ctx][hd/2][2] with the reference's cos/sin values */
void ember_host_rope_table(float *out, int ctx, int head_dim, float theta);

/* ---- extension on the public API (host C) ---- */
/* Greedy decoding on the device: equivalent to n iterations of
 *   logits = ember_forward(m, s, tok, pos + i); tok = first argmax(logits);
 * writing each chosen token to out_tokens[i]. The state's logits hold the last
 * step's logits afterwards. Returns s's logits. */
float *ember_forward_greedy(EmberModel *m, EmberState *s, int tok, int pos, int n,
                            int *out_tokens);
/* ember_sample(sampler, logits, vocab) for the logits of the state's last
 * ember_forward / ember_prefill, drawn on the device (no logits copied to the
 * host, no host sort). *rng_state is the sampler's xorshift64* state and
 * advances exactly as in the reference (one draw when temperature > 0);
 * history / hist_len are the sampler's history array and length (NULL / 0 when
 * it keeps none). As the reference's ember_sample would, the caller then records
 * the token with ember_sampler_accept. Returns the token; fatal errors follow the
 * library's convention. */
int ember_sample_device(EmberState *s, const EmberSampleParams *p, uint64_t *rng_state, const int *history,
                        int hist_len);
/* the device-side state behind a public state (for timing hooks) */
EmberCudaState *ember_state_cuda(EmberState *s);

/* Batched greedy decode of n_streams independent sequences on one model (see
 * ember_cuda_batch_*): prompts go in per stream, then every step advances all
 * streams at once. Fatal errors follow the library's convention (ember_die). */
typedef struct EmberBatch EmberBatch;
EmberBatch *ember_batch_new(EmberModel *m, int n_streams, int ctx_len, int kv_fp16, int max_steps);
void        ember_batch_free(EmberBatch *b);
/* the device-side batch behind a public batch (for timing hooks) */
EmberCudaBatch *ember_batch_cuda(EmberBatch *b);
/* prompt of stream `stream` at positions 0..n-1; returns its last token's logits
 * (vocab floats owned by the batch, valid until the next call) */
float      *ember_batch_prefill(EmberBatch *b, int stream, const int *ids, int n);
/* n_steps greedy steps: stream i feeds toks[i] at pos[i]; out_tokens (may be
 * NULL) [n_steps][n_streams]; out_logits (may be NULL) [n_streams][vocab] of the
 * last step */
void        ember_batch_greedy(EmberBatch *b, const int *toks, const int *pos, int n_steps, int *out_tokens,
                               float *out_logits);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* EMBER_B200_CUDA_H */
