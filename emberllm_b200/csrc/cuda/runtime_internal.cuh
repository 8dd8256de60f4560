// runtime_internal.cuh — the device-side model and run-state structures shared by
// the token-step runtime (runtime.cu) and the batched prefill (prefill.cu).
// Internal to the library: nothing here crosses the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <vector>

#include "ember_cuda.h"
#include "common.cuh"

namespace emb {

// Records a printf-style message for ember_cuda_error() and returns 1.
__attribute__((visibility("hidden"))) int set_err(const char *fmt, ...);

}  // namespace emb

#define CK(call)                                                                           \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return emb::set_err("%s (%s:%d: %s)", cudaGetErrorString(e_), __FILE__, __LINE__, #call); \
    } while (0)

// One weight matrix on the device. Quantized: q = [rows][cols/32] blocks of 32
// int8 (Q8_0) or 16 nibble bytes (Q4_0), row-major and contiguous; s = the fp16
// block scales [rows][cols/32] (padded by 256 bytes). fp32: q = [rows][cols].
struct DevMat {
    int dtype = EMBER_DT_F32, rows = 0, cols = 0;
    uint8_t *q = nullptr;
    __half *s = nullptr;
};

struct DevLayer {
    DevMat wq, wk, wv, wo, w1, w2, w3;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

namespace emb {
struct PfModel;   // batched-prefill weight packs (prefill.cu), built on first use
struct PfState;   // batched-prefill activations (prefill.cu), built on first use
struct PState;    // the persistent token step's plan and hand-off buffers (persist.cu)
struct SampleBufs;  // device sampling scratch (sample.cu), built on first use
}  // namespace emb

struct EmberCudaModel {
    int device = 0, n_sm = 148;
    int dim = 0, hidden = 0, n_layers = 0, n_heads = 0, n_kv = 0, head_dim = 0, vocab = 0;
    int qk_norm = 0, rope_neox = 0;
    float eps = 0;
    DevMat tok_emb, lm_head;
    float *final_norm = nullptr;
    std::vector<DevLayer> layers;
    emb::ExpfDev ex;
    std::vector<void *> allocs;
    uint64_t bytes = 0;
    emb::PfModel *pf = nullptr;
};

static inline int dalloc(EmberCudaModel *m, void **p, size_t n) {
    CK(cudaMalloc(p, n ? n : 16));
    m->allocs.push_back(*p);
    m->bytes += n;
    return 0;
}

struct EmberCudaState {
    EmberCudaModel *m = nullptr;
    int ctx = 0, kv_fp16 = 0, kstride = 0;
    cudaStream_t stream = nullptr;
    std::vector<void *> allocs;
    // device buffers
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *od = nullptr, *of = nullptr, *hd = nullptr, *hf = nullptr, *logits = nullptr;
    int8_t *oq = nullptr, *hq = nullptr;
    void *kc = nullptr, *vc = nullptr;
    size_t k_layer_elems = 0, v_layer_elems = 0;
    float2 *rope = nullptr;
    int *ctl = nullptr, *ids = nullptr, *out_tokens = nullptr;
    float *am_v = nullptr;
    int *am_i = nullptr;
    unsigned *am_ticket = nullptr;
    int am_blocks = 0;
    int att_in_smem = 0, attn_chunk = 0;
    size_t attn_smem = 0;
    int attn_split = 0, attn_splits = 1;   // split decode attention (attn_split.cuh)
    int attn_w_smem = 0;                   // softmax weights held in shared memory
    float *pmax = nullptr;
    int att_stride = 0;                    // row stride of att (ctx rounded up to 4)
    float *wglob = nullptr;                // softmax weights when they do not fit smem
    std::vector<CUtensorMap> kmaps;        // per layer: keys as [n_kv*hd][kstride], [hd][AS_PER] boxes
    std::vector<CUtensorMap> vmaps;        // per layer: values as [n_kv*ctx][hd], [AS_VB][32] boxes
    // pinned host
    float *h_logits = nullptr;
    int *h_ctl = nullptr;
    // graphs
    cudaGraphExec_t g_fwd = nullptr, g_greedy = nullptr, g_prefill = nullptr, g_head = nullptr;
    int launches_per_step = 0;
    int launches_greedy = 0;      // kernels of one device greedy token (0 until captured)
    emb::PfState *pf = nullptr;
    emb::PState *ps = nullptr;             // set when the persistent token step serves this state
    emb::SampleBufs *sb = nullptr;         // device sampling scratch
};

static inline int salloc(EmberCudaState *s, void **p, size_t n) {
    CK(cudaMalloc(p, n ? n : 16));
    s->allocs.push_back(*p);
    return 0;
}

// ember_cuda_prefill that always takes the batched path (also for one token)
int ember_cuda_prefill_batched(EmberCudaState *s, const int *ids, int n, int start, float *host_logits);
namespace emb {
// greedy decoding on a state's stream, split so that several states can run at once
int greedy_prepare(EmberCudaState *s);
int greedy_enqueue(EmberCudaState *s, int tok, int pos, int n_steps, int *host_tokens);
int greedy_finish(EmberCudaState *s);
}  // namespace emb

// ---- the persistent token step (persist.cu) ----
namespace emb {
// Sets s->ps when the state's model and context suit the persistent step
// (returns 0 and leaves s->ps NULL otherwise); 1 on a CUDA error.
int persist_init(EmberCudaState *s);
void persist_release(EmberCudaState *s);
// enqueue n_steps token steps from ctl's token and position on s->stream;
// greedy: pick between steps and write the picks to s->out_tokens
int persist_run(EmberCudaState *s, int n_steps, int greedy);
}  // namespace emb

// ---- device sampling (sample.cu) ----
namespace emb {
void sample_release(EmberCudaState *s);
}  // namespace emb

// ---- batched prefill (prefill.cu) ----
namespace emb {
// 1 when every layer matrix is Q8_0 / Q4_0 and the shapes suit the tensor-core
// path (otherwise prefill runs as exact single-token steps)
int pf_supported(const EmberCudaModel *m);
// Layers of tokens ids[0..n) (device array) at positions start.., the KV cache
// filled for them; leaves the last token's residual stream in s->x. Enqueued on
// s->stream.
int pf_run_layers(EmberCudaState *s, const int *ids_dev, int n, int start);
// 1 when a batched prefill of n tokens at `start` fits the attention tiling
int pf_fits(EmberCudaState *s, int n, int start);
void pf_model_release(EmberCudaModel *m);
void pf_state_release(EmberCudaState *s);
// tensor map of a 2-D fp32 / fp16 matrix [outer][inner] read in boxes of
// box_inner x box_outer elements (no swizzle)
int map_2d(CUtensorMap *map, const void *base, int elem_bytes, size_t inner, size_t outer, int box_inner,
           int box_outer);
// op level: out[B][d_out] = W x for B host columns through the tensor-core GEMM;
// xq_blocks (may be NULL) receives the columns' Q8_0 blocks
int pf_matmul_batch(int device, float *out, const float *x, const DevMat &w, int B, void *xq_blocks);
}  // namespace emb
