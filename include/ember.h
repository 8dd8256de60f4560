/* ember.h — the C-ABI boundary of the B200 token-loop library (libember_b200.so).
 *
 * This header declares exactly the entry points emberllm's callers bind: its CLI
 * (src/main.c), its HTTP server (src/server.c) and its ctypes bindings
 * (bindings/python/emberllm.py:89-109). Names, argument meaning, struct layouts
 * and the fatal-error convention are those of emberllm's public header
 * (src/ember.h:111-171); each declaration below cites the reference entry it
 * replaces. Callers compiled against emberllm's own src/ember.h link against this
 * library unchanged, because every struct here is layout-identical (checked by the
 * static asserts at the bottom).
 *
 * What runs where:
 *   - the .ember file is mmap'd on the host and validated exactly as emberllm does;
 *   - the first state created for a model uploads its weights to the GPU
 *     (repacked into a device layout, see emberllm_b200/csrc/cuda/);
 *   - ember_forward / ember_prefill run entirely on the GPU and hand back a
 *     pinned HOST float buffer of vocab_size logits owned by the state.
 * There is no CPU fallback: with no usable CUDA device, state creation ends the
 * process through ember_die ("ember: cuda: ...").
 *
 * Tokenizer and sampler entry points (emberllm src/ember.h:131-168) are host
 * text/policy code outside the token loop and are not part of this library; a
 * drop-in build links emberllm's own tokenizer.c / sample.c against it (see the
 * integration notes shipped with this repository).
 *
 * On-disk format (unchanged from emberllm, src/ember.h:1-14):
 *   [EmberHeader 256 B][tokenizer blob][tensor table, 8-aligned][pad][tensor data,
 *   each tensor 64-aligned]; all integers little-endian; 2-D tensors are
 *   [out_rows, in_len] row-major; Q8_0 rows are in_len/32 blocks of
 *   {fp16 d; int8 qs[32]} (34 B), Q4_0 rows are blocks of {fp16 d; u8 qs[16]}
 *   (18 B, byte i holds element i in its low nibble and element i+16 in its high
 *   nibble, values stored +8).
 */
#ifndef EMBER_B200_EMBER_H
#define EMBER_B200_EMBER_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* "EMBR" read as a little-endian u32, and the only format version (ref src/ember.h:21-22) */
#define EMBER_MAGIC   0x52424d45u
#define EMBER_VERSION 1u

/* stored tensor encodings (ref src/ember.h:25-30) */
enum {
    EMBER_DT_F32  = 0,
    EMBER_DT_Q8_0 = 1,
    EMBER_DT_Q4_0 = 2,
    EMBER_DT_F16  = 3
};

/* header flag bits (ref src/ember.h:33-37) */
enum {
    EMBER_FLAG_TIED_EMBED = 1u << 0,
    EMBER_FLAG_QK_NORM    = 1u << 1,
    EMBER_FLAG_THINKING   = 1u << 2
};

/* rotary pairing (ref src/ember.h:40-43): interleaved pairs (2i, 2i+1), or NEOX
 * half-split pairs (i, i + head_dim/2) */
enum {
    EMBER_ROPE_INTERLEAVED = 0,
    EMBER_ROPE_NEOX        = 1
};

/* tokenizer blob kinds (ref src/ember.h:46-49) */
enum {
    EMBER_TOK_LLAMA_SP = 0,
    EMBER_TOK_BYTE_BPE = 1
};

#define EMBER_Q_BLOCK 32

#pragma pack(push, 1)
/* 256-byte file header (ref src/ember.h:53-83). Field order and widths are the
 * file format and therefore identical to emberllm's. */
typedef struct {
    char     magic[4];
    uint32_t version;
    uint64_t header_bytes;         /* start of the tensor-data region              */
    int32_t  dim;
    int32_t  hidden_dim;
    int32_t  n_layers;
    int32_t  n_heads;
    int32_t  n_kv_heads;
    int32_t  head_dim;
    int32_t  vocab_size;
    int32_t  max_seq_len;
    float    rope_theta;
    float    norm_eps;
    uint32_t flags;
    int32_t  rope_style;
    int32_t  bos_token_id;
    int32_t  eos_token_id;
    int32_t  eos_token_id2;
    int32_t  n_tensors;
    int32_t  tokenizer_type;
    int32_t  default_top_k;
    float    default_temp;
    float    default_top_p;
    uint64_t tokenizer_offset;
    uint64_t tokenizer_size;
    uint64_t tensor_table_offset;
    uint64_t tensor_table_size;
    uint8_t  reserved[128];
} EmberHeader;

/* 88-byte tensor-table entry (ref src/ember.h:85-92) */
typedef struct {
    char     name[48];
    int32_t  dtype;
    int32_t  ndim;
    int32_t  shape[4];
    uint64_t offset;
    uint64_t nbytes;
} EmberTensor;
#pragma pack(pop)

typedef struct EmberModel     EmberModel;
typedef struct EmberTokenizer EmberTokenizer;
typedef struct EmberState     EmberState;

/* ---- model file (replaces ref src/io.c:30-96, declared at src/ember.h:112-117) ---- */

/* mmap + validate; NULL (with "ember: <why>" on stderr) on a bad file. Same checks
 * and order as ref src/io.c:30-72. No GPU work happens here. */
EmberModel        *ember_model_load(const char *path);
/* unmap, and release the model's device weights if a state uploaded them */
void               ember_model_free(EmberModel *m);
const EmberHeader *ember_model_header(const EmberModel *m);
/* first table entry whose 48-byte name equals `name`; NULL if absent (ref src/io.c:83-90) */
const EmberTensor *ember_model_tensor(const EmberModel *m, const char *name);
/* host pointer into the mapping; NULL if the tensor runs past the file (ref src/io.c:92-96) */
const void        *ember_model_data(const EmberModel *m, const EmberTensor *t);

/* ---- run state and the token loop (replaces ref src/model.c:116-414) ---- */

/* ref src/model.c:116-118: fp32 KV cache */
EmberState *ember_state_new(const EmberModel *m, int ctx_len);
/* ref src/model.c:120-193: resolves every tensor (dies naming the first missing
 * one), uploads the model to the GPU on first use, allocates the device KV cache
 * (fp16 when kv_fp16 != 0) and activations, and a pinned host logits buffer.
 * ctx_len <= 0 or >= max_seq_len selects max_seq_len, as in the reference. */
EmberState *ember_state_new_ex(const EmberModel *m, int ctx_len, int kv_fp16);
void        ember_state_free(EmberState *s);

/* ref src/model.c:362-414: one decode step for `tok` at `pos`. Returns the state's
 * host logits (vocab_size floats), valid until the next call on this state; the
 * caller may modify them. Dies on tok outside [0,vocab) or pos outside [0,ctx). */
float *ember_forward(EmberModel *m, EmberState *s, int tok, int pos);

/* ref src/model.c:283-360: ids[0..n) at positions start..start+n-1; fills the KV
 * cache and returns the LAST token's logits. n <= 0 returns the logits buffer
 * untouched. Dies on an out-of-range id, and (unlike the reference, which would
 * write past its cache) on start < 0 or start + n > ctx. */
float *ember_prefill(EmberModel *m, EmberState *s, const int *ids, int n, int start);

/* ---- offline requantizer (replaces ref src/quant.c:59-125) ---- */

/* fp32 .ember -> Q8_0 / Q4_0 .ember with the reference's rules and byte layout:
 * 1-D tensors stay fp32, rows not divisible by 32 stay fp32, and in Q4_0 mode the
 * tok_embeddings / lm_head tables stay Q8_0. Returns 0 on success. Host only. */
int ember_quantize_file(const char *in_path, const char *out_path, int target);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#ifndef __cplusplus
_Static_assert(sizeof(EmberHeader) == 256, "EmberHeader must stay 256 bytes");
_Static_assert(sizeof(EmberTensor) == 88, "EmberTensor must stay 88 bytes");
#else
static_assert(sizeof(EmberHeader) == 256, "EmberHeader must stay 256 bytes");
static_assert(sizeof(EmberTensor) == 88, "EmberTensor must stay 88 bytes");
#endif

#endif /* EMBER_B200_EMBER_H */
