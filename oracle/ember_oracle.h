/* ember_oracle.h — TEST INFRASTRUCTURE ONLY. A plain-C restatement of emberllm's
 * token loop used as the parity checker for the GPU library. Nothing in the
 * product (emberllm_b200/) links, loads or calls this code; only tests/, the
 * smoke check and bench.py's CPU-baseline leg do.
 *
 * Parity pin: tests/test_oracle_pin.py checks this restatement bit for bit
 * against the unmodified reference compiled from its own sources
 * (oracle/_ref/libember_ref_det.so, built by oracle/Makefile) on synthetic
 * models, and against the committed golden vectors in tests/golden/.
 */
#ifndef EMBER_ORACLE_H
#define EMBER_ORACLE_H

#include <stdint.h>

typedef struct OrcModel OrcModel;
typedef struct OrcState OrcState;

OrcModel *orc_load(const char *path);
void      orc_free(OrcModel *m);
OrcState *orc_state_new(OrcModel *m, int ctx_len, int kv_fp16);
void      orc_state_free(OrcState *s);
int       orc_state_ctx(const OrcState *s);
float    *orc_forward(OrcState *s, int tok, int pos);
float    *orc_prefill(OrcState *s, const int *ids, int n, int start);
int       orc_argmax(const float *v, int n);

/* op level: same contracts as the reference's ember_matmul / quantize_q8_0 */
void orc_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out,
                void *xq_blocks);
void orc_matmul_batch(float *out, const float *x, const void *w, int dtype, int n_in,
                      int d_out, int B, void *xq_blocks);
void orc_quantize_q8_0(const float *x, void *out_blocks, int n);
void orc_quantize_q4_0(const float *x, void *out_blocks, int n);
uint16_t orc_f32_to_f16(float f);
float    orc_f16_to_f32(uint16_t h);
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
float orc_expf(float x);
void orc_set_threads(int n);
/* the reference's sampler over host logits (modified in place); *rng advances */
int orc_sample(float *logits, int n, float temperature, float top_p, int top_k, float min_p,
               float repeat_penalty, float presence_penalty, float frequency_penalty, uint64_t *rng,
               const int *hist, int hist_len);

#endif
