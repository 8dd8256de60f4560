// runtime.cu — the ember_cuda_* shim: device weights, run states, the captured
// token-step graphs, and the op-level ember_matmul entry points.
//
// Device layout. A .ember Q8_0 row is an array of 34-byte {fp16 d; int8 qs[32]}
// blocks (18-byte for Q4_0), so rows are not 16-byte aligned and scales sit
// between the quants. At upload every quantized matrix is split into a
// row-major byte array (32 or 16 bytes per block, every row 16-byte aligned) and
// a separate [rows][cols/32] fp16 scale array; a tile of R consecutive rows is
// then two contiguous byte ranges, each moved by one bulk copy. The KV cache is
// per layer and kv head: keys TRANSPOSED, [hd][kstride] (kstride = ctx rounded
// up to 8), so one thread per position reads consecutive addresses per
// dimension; values [ctx][hd].
//
// Execution. One token step is a fixed sequence of kernels (kernels.cuh) that
// read the position and token from device memory, captured once per state into
// CUDA graphs and replayed for every token. Kernels are launched with
// programmatic stream serialization so each one starts while its predecessor
// finishes and pulls its own weights into shared memory before waiting on the
// data it needs.
#include <cuda_runtime.h>

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "ember_cuda.h"
#include "ember_ops.h"
#include "kernels.cuh"
#include "attn_split.cuh"
#include "head.cuh"
#include "runtime_internal.cuh"

using namespace emb;

// ------------------------------------------------------------------ errors ----

static char g_err[512] = "no error";

namespace emb {
int set_err(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return 1;
}
}  // namespace emb

extern "C" const char *ember_cuda_error(void) { return g_err; }

static int pick_device(int *dev) {
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (n <= 0) return set_err("no CUDA device is visible");
    const char *env = getenv("EMBER_CUDA_DEVICE");
    int d = env && *env ? atoi(env) : 0;
    if (d < 0 || d >= n) return set_err("EMBER_CUDA_DEVICE=%d but %d device(s) are visible", d, n);
    CK(cudaSetDevice(d));
    cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, d));
    if (p.major < 10) return set_err("device %d (%s) is sm_%d%d; this library is built for sm_100a", d, p.name, p.major, p.minor);
    *dev = d;
    return 0;
}

extern "C" int ember_cuda_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) { cudaGetLastError(); return 0; }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) return 0;
    return p.major >= 10;
}

// Raise the dynamic shared-memory limit of every kernel instantiation once per
// device, outside any stream capture.
// each kernel may use the device's opt-in maximum minus its own static smem
template <typename K>
static int allow_max_smem(K kernel, int optin) {
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, kernel));
    CK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes));
    return 0;
}

static int init_kernel_attrs(int device) {
    static unsigned done_mask = 0;
    if (device < 32 && ((done_mask >> device) & 1u)) return 0;
    int optin = 0;
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    if (allow_max_smem(ember_q8_gemv_kernel<IN_RAW, EPI_STORE>, optin) || allow_max_smem(ember_q8_gemv_kernel<IN_NORM, EPI_STORE>, optin) ||
        allow_max_smem(ember_q8_gemv_kernel<IN_NORM, EPI_SWIGLU>, optin) || allow_max_smem(ember_q8_gemv_kernel<IN_QUANT, EPI_RESID>, optin) ||
        allow_max_smem(attn_decode_kernel<float>, optin) || allow_max_smem(attn_decode_kernel<__half>, optin) ||
        allow_max_smem(attn_scores_kernel<float, 1>, optin) || allow_max_smem(attn_scores_kernel<__half, 1>, optin) ||
        allow_max_smem(attn_scores_kernel<float, 2>, optin) || allow_max_smem(attn_scores_kernel<__half, 2>, optin) ||
        allow_max_smem(attn_scores_kernel<float, 4>, optin) || allow_max_smem(attn_scores_kernel<__half, 4>, optin) ||
        allow_max_smem(attn_scores_kernel<float, 8>, optin) || allow_max_smem(attn_scores_kernel<__half, 8>, optin) ||
        allow_max_smem(attn_softmax_pv_kernel<float, true>, optin) ||
        allow_max_smem(attn_softmax_pv_kernel<__half, true>, optin) ||
        allow_max_smem(attn_softmax_pv_kernel<float, false>, optin) ||
        allow_max_smem(attn_softmax_pv_kernel<__half, false>, optin) ||
        allow_max_smem(lm_head_kernel<false, false>, optin) || allow_max_smem(lm_head_kernel<true, false>, optin) ||
        allow_max_smem(lm_head_kernel<false, true>, optin) || allow_max_smem(lm_head_kernel<true, true>, optin))
        return 1;
    if (device < 32) done_mask |= 1u << device;
    return 0;
}

// ------------------------------------------------------------------ model -----

static int upload_vec(EmberCudaModel *m, float **dst, const float *src, int n) {
    if (!src) { *dst = nullptr; return 0; }
    if (dalloc(m, (void **)dst, (size_t)n * 4)) return 1;
    CK(cudaMemcpy(*dst, src, (size_t)n * 4, cudaMemcpyHostToDevice));
    return 0;
}

// Split AoS blocks into quant rows + scale rows and upload. The scale array is
// padded by 256 bytes: tile copies round their size up to 16 bytes.
static int upload_mat(EmberCudaModel *m, DevMat *d, const EmberCudaMat &h) {
    d->dtype = h.dtype;
    d->rows = h.rows;
    d->cols = h.cols;
    const size_t rows = (size_t)h.rows;
    if (h.dtype == EMBER_DT_F32) {
        size_t n = rows * h.cols * 4;
        if (dalloc(m, (void **)&d->q, n)) return 1;
        CK(cudaMemcpy(d->q, h.data, n, cudaMemcpyHostToDevice));
        return 0;
    }
    const int nb = h.cols / 32;
    const size_t blk_in = h.dtype == EMBER_DT_Q8_0 ? 34 : 18, blk_q = blk_in - 2;
    const size_t qn = rows * nb * blk_q, sn = rows * nb * 2;
    if (dalloc(m, (void **)&d->q, qn) || dalloc(m, (void **)&d->s, sn + 256)) return 1;
    CK(cudaMemset(d->s, 0, sn + 256));
    const size_t chunk_rows = 4096;
    std::vector<uint8_t> qb(chunk_rows * nb * blk_q);
    std::vector<uint16_t> sb(chunk_rows * nb);
    const uint8_t *src = (const uint8_t *)h.data;
    for (size_t r0 = 0; r0 < rows; r0 += chunk_rows) {
        size_t nr = rows - r0 < chunk_rows ? rows - r0 : chunk_rows;
        for (size_t r = 0; r < nr; r++)
            for (int b = 0; b < nb; b++) {
                const uint8_t *blk = src + ((r0 + r) * nb + b) * blk_in;
                memcpy(&sb[r * nb + b], blk, 2);
                memcpy(&qb[(r * nb + b) * blk_q], blk + 2, blk_q);
            }
        CK(cudaMemcpy(d->q + r0 * nb * blk_q, qb.data(), nr * nb * blk_q, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(d->s + r0 * nb, sb.data(), nr * nb * 2, cudaMemcpyHostToDevice));
    }
    return 0;
}

static void model_release(EmberCudaModel *m) {
    pf_model_release(m);
    for (void *p : m->allocs) cudaFree(p);
    m->allocs.clear();
}

extern "C" int ember_cuda_model_upload(const EmberCudaModelDesc *d, const EmberExpfParams *e,
                                       EmberCudaModel **out) {
    *out = nullptr;
    EmberCudaModel *m = new EmberCudaModel();
    int rc = pick_device(&m->device);
    if (rc) { delete m; return rc; }
    int nsm = 0;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, m->device);
    m->n_sm = nsm > 0 ? nsm : 148;
    m->dim = d->dim; m->hidden = d->hidden; m->n_layers = d->n_layers; m->n_heads = d->n_heads;
    m->n_kv = d->n_kv_heads; m->head_dim = d->head_dim; m->vocab = d->vocab; m->qk_norm = d->qk_norm;
    m->rope_neox = d->rope_neox;
    m->eps = d->norm_eps;
    const int hd = d->head_dim, qd = d->n_heads * hd, kvd = d->n_kv_heads * hd;
    m->layers.resize(d->n_layers);
    rc = upload_mat(m, &m->tok_emb, d->tok_emb);
    if (!rc) {
        if (d->lm_head.data == d->tok_emb.data) m->lm_head = m->tok_emb;   // tied: one copy
        else rc = upload_mat(m, &m->lm_head, d->lm_head);
    }
    if (!rc) rc = upload_vec(m, &m->final_norm, d->final_norm, d->dim);
    for (int l = 0; l < d->n_layers && !rc; l++) {
        DevLayer &L = m->layers[l];
        rc = upload_mat(m, &L.wq, d->wq[l]) || upload_mat(m, &L.wk, d->wk[l]) ||
             upload_mat(m, &L.wv, d->wv[l]) || upload_mat(m, &L.wo, d->wo[l]) ||
             upload_mat(m, &L.w1, d->w1[l]) || upload_mat(m, &L.w2, d->w2[l]) ||
             upload_mat(m, &L.w3, d->w3[l]) ||
             upload_vec(m, &L.attn_norm, d->attn_norm[l], d->dim) ||
             upload_vec(m, &L.ffn_norm, d->ffn_norm[l], d->dim) ||
             upload_vec(m, &L.q_norm, d->q_norm[l], hd) || upload_vec(m, &L.k_norm, d->k_norm[l], hd) ||
             upload_vec(m, &L.bq, d->b_q[l], qd) || upload_vec(m, &L.bk, d->b_k[l], kvd) ||
             upload_vec(m, &L.bv, d->b_v[l], kvd);
    }
    if (!rc) {
        // the expf recipe's 2^(j/64) table, then the exception slots
        m->ex.p = *e;
        double *tab = nullptr;
        uint32_t *slots = nullptr;
        rc = dalloc(m, (void **)&tab, 64 * sizeof(double)) || dalloc(m, (void **)&slots, (size_t)e->n_slots * 8);
        if (!rc && (cudaMemcpy(tab, e->tab, 64 * sizeof(double), cudaMemcpyHostToDevice) != cudaSuccess ||
                    cudaMemcpy(slots, e->slots, (size_t)e->n_slots * 8, cudaMemcpyHostToDevice) != cudaSuccess))
            rc = set_err("expf table upload failed");
        m->ex.p.tab = tab;
        m->ex.p.slots = slots;
    }
    if (rc) { model_release(m); delete m; return 1; }
    *out = m;
    return 0;
}

extern "C" void ember_cuda_model_free(EmberCudaModel *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    model_release(m);
    delete m;
}

extern "C" uint64_t ember_cuda_model_bytes(const EmberCudaModel *m) { return m ? m->bytes : 0; }

// ------------------------------------------------------------------ state -----

static void state_release(EmberCudaState *s) {
    pf_state_release(s);
    persist_release(s);
    sample_release(s);
    if (s->g_fwd) cudaGraphExecDestroy(s->g_fwd);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    if (s->g_prefill) cudaGraphExecDestroy(s->g_prefill);
    if (s->g_head) cudaGraphExecDestroy(s->g_head);
    for (void *p : s->allocs) cudaFree(p);
    s->allocs.clear();
    if (s->h_logits) cudaFreeHost(s->h_logits);
    if (s->h_ctl) cudaFreeHost(s->h_ctl);
    if (s->stream) cudaStreamDestroy(s->stream);
}

extern "C" int ember_cuda_state_new(EmberCudaModel *m, int ctx, int kv_fp16, const float *rope_cs,
                                    EmberCudaState **out) {
    *out = nullptr;
    CK(cudaSetDevice(m->device));
    if (init_kernel_attrs(m->device)) return 1;
    EmberCudaState *s = new EmberCudaState();
    s->m = m;
    s->ctx = ctx;
    s->kv_fp16 = kv_fp16;
    s->kstride = (ctx + 7) / 8 * 8;
    const int hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
    const size_t es = kv_fp16 ? 2 : 4;
    s->k_layer_elems = (size_t)m->n_kv * hd * s->kstride;
    s->v_layer_elems = (size_t)m->n_kv * ctx * hd;
    const size_t k_bytes = (size_t)m->n_layers * s->k_layer_elems * es + 256;
    const size_t v_bytes = (size_t)m->n_layers * s->v_layer_elems * es + 256;
    s->am_blocks = m->n_sm;
    // attention shared memory: two chunk buffers (keys/values of `attn_chunk`
    // cached positions each) and, when they fit, the scores of all positions
    {
        const size_t budget = 200 * 1024, att_bytes = pad16((size_t)ctx * 4);
        s->att_in_smem = att_bytes <= 48 * 1024;
        const size_t for_bufs = budget - (s->att_in_smem ? att_bytes : 0);
        int chunk = (int)(for_bufs / (2 * (size_t)hd * es)) / 8 * 8;
        if (chunk > 1024) chunk = 1024;
        if (chunk < 8) chunk = 8;
        s->attn_chunk = chunk;
        s->attn_smem = 2 * (size_t)chunk * hd * es + (s->att_in_smem ? att_bytes : 0);
    }
    int rc = 0;
    rc |= salloc(s, (void **)&s->x, (size_t)m->dim * 4);
    rc |= salloc(s, (void **)&s->q, (size_t)qd * 4);
    rc |= salloc(s, (void **)&s->k, (size_t)kvd * 4);
    rc |= salloc(s, (void **)&s->v, (size_t)kvd * 4);
    // split attention (attn_split.cuh): AS_PER cached positions per scoring CTA;
    // the softmax weights sit in shared memory when they fit
    // Short contexts keep the single-kernel attention (one launch fewer per layer);
    // longer ones split the cache over CTAs. The crossover scales with the work per
    // position: 512 positions at head_dim 128 (Qwen3 at 1160: split 721 tok/s, fused
    // 563), 1024 at head_dim 64 and below (Qwen2.5 at 648: fused 987 against 723;
    // SmolLM2 at 776: 937 against 870). EMBER_ATTN=fused / split forces one.
    const char *attn_env = getenv("EMBER_ATTN");
    const bool force_fused = attn_env && strcmp(attn_env, "fused") == 0;
    const bool force_split = attn_env && strcmp(attn_env, "split") == 0;
    const int split_above = hd <= 64 ? 1024 : 512;
    s->attn_split = m->n_heads / m->n_kv <= AS_MAX_KVMUL && hd <= 256 && hd % 32 == 0 && !force_fused &&
                    (force_split || ctx > split_above);
    s->attn_splits = (ctx + AS_PER - 1) / AS_PER;
    s->attn_w_smem = as_pv_smem(m->n_heads / m->n_kv, ctx, (int)es, 1) <= 200 * 1024;
    s->att_stride = (ctx + 63) / 64 * 64;   // split_chain_sum pads rows to 64 positions
    rc |= salloc(s, (void **)&s->att, (size_t)m->n_heads * s->att_stride * 4 + 256);
    if (s->attn_split && !s->attn_w_smem)
        rc |= salloc(s, (void **)&s->wglob, (size_t)(hd / 32) * m->n_heads * s->att_stride * 4 + 256);
    rc |= salloc(s, (void **)&s->pmax, (size_t)m->n_heads * s->attn_splits * 4);
    rc |= salloc(s, (void **)&s->oq, (size_t)qd + 16);
    rc |= salloc(s, (void **)&s->od, (size_t)qd / 32 * 4 + 16);
    rc |= salloc(s, (void **)&s->of, (size_t)qd * 4);
    rc |= salloc(s, (void **)&s->hq, (size_t)m->hidden + 16);
    rc |= salloc(s, (void **)&s->hd, (size_t)m->hidden / 32 * 4 + 16);
    rc |= salloc(s, (void **)&s->hf, (size_t)m->hidden * 4);
    rc |= salloc(s, (void **)&s->logits, (size_t)m->vocab * 4);
    rc |= salloc(s, &s->kc, k_bytes);
    rc |= salloc(s, &s->vc, v_bytes);
    rc |= salloc(s, (void **)&s->rope, (size_t)ctx * (hd / 2) * sizeof(float2));
    rc |= salloc(s, (void **)&s->ctl, CTL_WORDS * 4);
    rc |= salloc(s, (void **)&s->ids, (size_t)ctx * 4);
    rc |= salloc(s, (void **)&s->out_tokens, (size_t)ctx * 4 + 4);
    rc |= salloc(s, (void **)&s->am_v, (size_t)s->am_blocks * 4);
    rc |= salloc(s, (void **)&s->am_i, (size_t)s->am_blocks * 4);
    rc |= salloc(s, (void **)&s->am_ticket, 4);
    if (rc) { state_release(s); delete s; return 1; }
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMallocHost(&s->h_logits, (size_t)m->vocab * 4) != cudaSuccess ||
        cudaMallocHost(&s->h_ctl, CTL_WORDS * 4) != cudaSuccess) {
        set_err("stream / pinned host allocation failed: %s", cudaGetErrorString(cudaGetLastError()));
        state_release(s);
        delete s;
        return 1;
    }
    memset(s->h_ctl, 0, CTL_WORDS * 4);
    if (cudaMemcpy(s->rope, rope_cs, (size_t)ctx * (hd / 2) * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(s->kc, 0, k_bytes) != cudaSuccess || cudaMemset(s->vc, 0, v_bytes) != cudaSuccess ||
        cudaMemset(s->ctl, 0, CTL_WORDS * 4) != cudaSuccess || cudaMemset(s->am_ticket, 0, 4) != cudaSuccess ||
        cudaMemset(s->logits, 0, (size_t)m->vocab * 4) != cudaSuccess) {
        set_err("state initialisation failed: %s", cudaGetErrorString(cudaGetLastError()));
        state_release(s);
        delete s;
        return 1;
    }
    memset(s->h_logits, 0, (size_t)m->vocab * 4);
    if (s->attn_split) {
        // per layer: the keys as one [n_kv*hd][kstride] matrix read in [hd][AS_PER]
        // boxes, the values as one [n_kv*ctx][hd] matrix read in [AS_VB][32] boxes
        s->kmaps.resize(m->n_layers);
        s->vmaps.resize(m->n_layers);
        for (int l = 0; l < m->n_layers; l++)
            if (map_2d(&s->kmaps[l], (char *)s->kc + (size_t)l * s->k_layer_elems * es, (int)es,
                       (size_t)s->kstride, (size_t)m->n_kv * hd, AS_PER, hd) ||
                map_2d(&s->vmaps[l], (char *)s->vc + (size_t)l * s->v_layer_elems * es, (int)es, (size_t)hd,
                       (size_t)m->n_kv * ctx, 32, AS_VB)) {
                state_release(s);
                delete s;
                return 1;
            }
    }
    // the token step as one persistent kernel where the model and context suit it
    if (persist_init(s)) {
        state_release(s);
        delete s;
        return 1;
    }
    *out = s;
    return 0;
}

extern "C" void ember_cuda_state_free(EmberCudaState *s) {
    if (!s) return;
    cudaSetDevice(s->m->device);
    if (s->stream) cudaStreamSynchronize(s->stream);
    state_release(s);
    delete s;
}

extern "C" float *ember_cuda_state_host_logits(EmberCudaState *s) { return s->h_logits; }
extern "C" void *ember_cuda_state_stream(EmberCudaState *s) { return (void *)s->stream; }
extern "C" const float *ember_cuda_state_logits_dev(EmberCudaState *s) { return s->logits; }
extern "C" int ember_cuda_state_launches_per_step(const EmberCudaState *s) { return s->launches_per_step; }
extern "C" int ember_cuda_state_launches_per_token(const EmberCudaState *s) { return s->launches_greedy; }

// ------------------------------------------------------------------ launches --

// Profiling hook: when set, every launch of a step records an event first, so
// ember_cuda_profile_step can report per-launch device times (no PDL overlap).
static cudaEvent_t *g_prof_events = nullptr;
static int g_prof_n = 0, g_prof_cap = 0;

// EMBER_PDL=0 launches without programmatic dependent launch (for comparisons)
static bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("EMBER_PDL");
        v = (e && *e == '0') ? 0 : 1;
    }
    return v == 1;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int block, size_t smem, cudaStream_t st,
                              Args... args) {
    if (g_prof_events && g_prof_n < g_prof_cap) {
        cudaError_t e = cudaEventRecord(g_prof_events[g_prof_n++], st);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3((unsigned)block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl_enabled() && !g_prof_events) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

static GemvSeg seg_of(const DevMat &d, float *out, const float *bias) {
    GemvSeg g;
    g.q = d.q;
    g.s = d.s;
    g.dtype = d.dtype;
    g.rows = d.rows;
    g.out = out;
    g.bias = bias;
    return g;
}

// Choose the tile height, ring depth and grid of one gemv launch and launch it.
// Segments must agree on being quantized (callers split otherwise).
// max_ctas > 0 caps the grid of a non-persistent launch (taller tiles) so that
// SMs stay free for the next kernel's CTAs to start early.
template <int IN, int EPI>
static int run_gemv(GemvArgs a, int n_sm, cudaStream_t st, int *count, int max_ctas = 0) {
    const int nsub = EPI == EPI_SWIGLU ? 2 : 1;
    a.quantized = a.seg[0].dtype != EMBER_DT_F32;
    int rows_total = 0;
    for (int k = 0; k < a.nseg; k++) rows_total += a.seg[k].rows;
    // SwiGLU tiles are one quant block of h (32 rows); others shrink to spread
    // small matrices over more SMs (R >= 8 keeps scale copies 16-byte aligned)
    int R = GEMV_MAX_ROWS;
    if (EPI != EPI_SWIGLU) {
        while (R > 8 && (rows_total + R - 1) / R < n_sm) R /= 2;
        while (max_ctas > 0 && R < GEMV_MAX_ROWS && (rows_total + R - 1) / R > max_ctas) R *= 2;
    }
    a.rows = R;
    if (EPI == EPI_SWIGLU) {
        a.tiles[0] = 0;
        a.tiles[1] = a.tiles[2] = a.tiles[3] = (a.seg[0].rows + R - 1) / R;
        a.nseg = 1;   // tiles[nseg] counts pairs; both matrices are read per tile
    } else {
        a.tiles[0] = 0;
        for (int k = 0; k < a.nseg; k++) a.tiles[k + 1] = a.tiles[k] + (a.seg[k].rows + R - 1) / R;
        for (int k = a.nseg + 1; k < 4; k++) a.tiles[k] = a.tiles[a.nseg];
    }
    const int total = a.tiles[a.nseg];
    size_t sb = 0;
    for (int sub = 0; sub < nsub; sub++) sb += gemv_sub_bytes(a.seg[sub].dtype, R, a.cols);
    a.stage_bytes = (int)((sb + 127) / 128 * 128);
    // Grid: every CTA resident at once (a second wave would double the time).
    // One CTA per tile when all tiles fit; otherwise a persistent grid with a
    // ring of 2-4 stages, choosing the depth that keeps the most bytes in flight
    // per SM (CTAs per SM x stages).
    const bool need_xf = IN != IN_QUANT || !a.quantized;
    auto resident = [&](int stages, size_t *smem_out) {
        a.stages = a.quantized ? stages : 0;
        size_t smem = gemv_smem_bytes(a, need_xf, IN == IN_NORM);
        *smem_out = smem;
        int occ = 0;
        if (smem > 200 * 1024 ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ember_q8_gemv_kernel<IN, EPI>, GEMV_THREADS, smem) != cudaSuccess)
            return 0;
        return occ;
    };
    size_t smem = 0;
    int grid = 0, best_stages = 1;
    const int occ1 = resident(1, &smem);
    if (occ1 <= 0) return set_err("gemv tile of %d x %d does not fit shared memory", R, a.cols);
    if (total <= occ1 * n_sm || !a.quantized) {
        grid = total < occ1 * n_sm ? total : occ1 * n_sm;
    } else {
        int best = 0;
        for (int s = 2; s <= GEMV_MAX_STAGES; s++) {
            size_t sm = 0;
            const int occ = resident(s, &sm);
            if (occ * s > best) { best = occ * s; best_stages = s; grid = occ * n_sm; }
        }
        if (best == 0) { best_stages = 1; grid = occ1 * n_sm; }
        if (grid > total) grid = total;
    }
    if (grid < 1) grid = 1;
    resident(total <= grid ? 1 : best_stages, &smem);
    if (count) (*count)++;
    CK(launch_pdl(ember_q8_gemv_kernel<IN, EPI>, grid, GEMV_THREADS, smem, st, a));
    return 0;
}

static bool is_q(const DevMat &d) { return d.dtype != EMBER_DT_F32; }

// ---- the launches of a token step, one helper per kernel kind ----

enum { K_QKV = 0, K_ATTN = 1, K_WO = 2, K_W13 = 3, K_W2 = 4, K_HEAD = 5 };

static int launch_embed(EmberCudaState *s, const int *ids, int *count) {
    EmberCudaModel *m = s->m;
    EmbedArgs ea;
    ea.q = m->tok_emb.q; ea.s = m->tok_emb.s; ea.dtype = m->tok_emb.dtype; ea.dim = m->dim;
    ea.ctl = s->ctl; ea.ids = ids; ea.x = s->x;
    CK(launch_pdl(embed_kernel, 1, 256, 0, s->stream, ea));
    (*count)++;
    return 0;
}

static GemvArgs gemv_base(EmberCudaState *s) {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.ex = s->m->ex;
    a.err = s->ctl + CTL_ERR;
    return a;
}

static int launch_layer(EmberCudaState *s, int kind, int l, int *count) {
    EmberCudaModel *m = s->m;
    cudaStream_t st = s->stream;
    const DevLayer &L = m->layers[l];
    const int hd = m->head_dim;
    const size_t es = s->kv_fp16 ? 2 : 4;
    GemvArgs a = gemv_base(s);
    switch (kind) {
    case K_QKV:
        a.cols = m->dim;
        a.x = s->x; a.norm_w = L.attn_norm; a.eps = m->eps;
        if (is_q(L.wq) == is_q(L.wk) && is_q(L.wq) == is_q(L.wv)) {
            a.seg[0] = seg_of(L.wq, s->q, L.bq);
            a.seg[1] = seg_of(L.wk, s->k, L.bk);
            a.seg[2] = seg_of(L.wv, s->v, L.bv);
            a.nseg = 3;
            // the single-kernel attention that follows needs whole SMs (large
            // key/value buffers): leave one free per query head
            return run_gemv<IN_NORM, EPI_STORE>(a, m->n_sm, st, count,
                                                s->attn_split ? 0 : m->n_sm - m->n_heads);
        } else {
            const DevMat *mats[3] = { &L.wq, &L.wk, &L.wv };
            float *outs[3] = { s->q, s->k, s->v };
            const float *bias[3] = { L.bq, L.bk, L.bv };
            for (int j = 0; j < 3; j++) {
                a.seg[0] = seg_of(*mats[j], outs[j], bias[j]);
                a.nseg = 1;
                if (run_gemv<IN_NORM, EPI_STORE>(a, m->n_sm, st, count)) return 1;
            }
            return 0;
        }
    case K_ATTN: {
        if (s->attn_split) {
            AttnSplitArgs as;
            memset(&as, 0, sizeof(as));
            as.q = s->q; as.k = s->k; as.v = s->v;
            as.kc = (char *)s->kc + (size_t)l * s->k_layer_elems * es;
            as.vc = (char *)s->vc + (size_t)l * s->v_layer_elems * es;
            as.q_norm = L.q_norm; as.k_norm = L.k_norm;
            as.rope = s->rope; as.ctl = s->ctl; as.att = s->att; as.pmax = s->pmax; as.wglob = s->wglob;
            as.oq = s->oq; as.od = s->od; as.of = is_q(L.wo) ? nullptr : s->of;
            as.nh = m->n_heads; as.nkv = m->n_kv; as.hd = hd; as.ctx = s->ctx; as.kstride = s->kstride;
            as.neox = m->rope_neox; as.splits = s->attn_splits; as.w_smem = s->attn_w_smem;
            as.ast = s->att_stride; as.eps = m->eps; as.ex = m->ex;
            const dim3 g1((unsigned)m->n_kv, (unsigned)s->attn_splits), g2((unsigned)m->n_kv, (unsigned)(hd / 32));
            const size_t sm1 = as_scores_smem(hd, (int)es);
            const size_t sm2 = as_pv_smem(m->n_heads / m->n_kv, s->ctx, (int)es, s->attn_w_smem);
            const int kv_mul = m->n_heads / m->n_kv;
            const CUtensorMap &km = s->kmaps[l];
            if (s->kv_fp16) {
                if (kv_mul == 1) CK(launch_pdl(attn_scores_kernel<__half, 1>, g1, AS_THREADS, sm1, st, km, as));
                else if (kv_mul == 2) CK(launch_pdl(attn_scores_kernel<__half, 2>, g1, AS_THREADS, sm1, st, km, as));
                else if (kv_mul <= 4) CK(launch_pdl(attn_scores_kernel<__half, 4>, g1, AS_THREADS, sm1, st, km, as));
                else CK(launch_pdl(attn_scores_kernel<__half, 8>, g1, AS_THREADS, sm1, st, km, as));
                if (s->attn_w_smem) CK(launch_pdl(attn_softmax_pv_kernel<__half, true>, g2, AS_THREADS, sm2, st, s->vmaps[l], as));
                else CK(launch_pdl(attn_softmax_pv_kernel<__half, false>, g2, AS_THREADS, sm2, st, s->vmaps[l], as));
            } else {
                if (kv_mul == 1) CK(launch_pdl(attn_scores_kernel<float, 1>, g1, AS_THREADS, sm1, st, km, as));
                else if (kv_mul == 2) CK(launch_pdl(attn_scores_kernel<float, 2>, g1, AS_THREADS, sm1, st, km, as));
                else if (kv_mul <= 4) CK(launch_pdl(attn_scores_kernel<float, 4>, g1, AS_THREADS, sm1, st, km, as));
                else CK(launch_pdl(attn_scores_kernel<float, 8>, g1, AS_THREADS, sm1, st, km, as));
                if (s->attn_w_smem) CK(launch_pdl(attn_softmax_pv_kernel<float, true>, g2, AS_THREADS, sm2, st, s->vmaps[l], as));
                else CK(launch_pdl(attn_softmax_pv_kernel<float, false>, g2, AS_THREADS, sm2, st, s->vmaps[l], as));
            }
            (*count) += 2;
            return 0;
        }
        AttnArgs at;
        memset(&at, 0, sizeof(at));
        at.q = s->q; at.k = s->k; at.v = s->v;
        at.kc = (char *)s->kc + (size_t)l * s->k_layer_elems * es;
        at.vc = (char *)s->vc + (size_t)l * s->v_layer_elems * es;
        at.q_norm = L.q_norm; at.k_norm = L.k_norm;
        at.rope = s->rope; at.ctl = s->ctl; at.att = s->att;
        at.oq = s->oq; at.od = s->od; at.of = is_q(L.wo) ? nullptr : s->of;
        at.nh = m->n_heads; at.nkv = m->n_kv; at.hd = hd; at.ctx = s->ctx; at.kstride = s->kstride;
        at.neox = m->rope_neox; at.att_in_smem = s->att_in_smem; at.eps = m->eps; at.ex = m->ex;
        at.chunk = s->attn_chunk;
        if (s->kv_fp16) CK(launch_pdl(attn_decode_kernel<__half>, m->n_heads, ATTN_THREADS, s->attn_smem, st, at));
        else CK(launch_pdl(attn_decode_kernel<float>, m->n_heads, ATTN_THREADS, s->attn_smem, st, at));
        (*count)++;
        return 0;
    }
    case K_WO:
        a.cols = m->n_heads * hd;
        a.xq = s->oq; a.xd = s->od; a.xf = s->of;
        a.seg[0] = seg_of(L.wo, s->x, nullptr);
        a.nseg = 1;
        return run_gemv<IN_QUANT, EPI_RESID>(a, m->n_sm, st, count);
    case K_W13:
        if (is_q(L.w1) != is_q(L.w3)) return set_err("layer %d: w1 and w3 differ in quantization", l);
        a.cols = m->dim;
        a.x = s->x; a.norm_w = L.ffn_norm; a.eps = m->eps;
        a.seg[0] = seg_of(L.w1, nullptr, nullptr);
        a.seg[1] = seg_of(L.w3, nullptr, nullptr);
        a.nseg = 2;
        a.hq = s->hq; a.hd = s->hd; a.hf = is_q(L.w2) ? nullptr : s->hf;
        return run_gemv<IN_NORM, EPI_SWIGLU>(a, m->n_sm, st, count);
    case K_W2:
        a.cols = m->hidden;
        a.xq = s->hq; a.xd = s->hd; a.xf = s->hf;
        a.seg[0] = seg_of(L.w2, s->x, nullptr);
        a.nseg = 1;
        return run_gemv<IN_QUANT, EPI_RESID>(a, m->n_sm, st, count);
    }
    return set_err("unknown kernel kind %d", kind);
}

// The streaming lm_head kernel (head.cuh) for a Q8_0 / Q4_0 head of at most 32
// blocks per row; its ring takes as many stages as shared memory holds (at
// least two). Returns the depth, or 0 when the head keeps the tiled GEMV.
template <bool ARGMAX, bool Q4>
static int head_stages(int device, int stage_bytes, int cols) {
    static int optin[32] = {0};
    if (device < 0 || device >= 32) return 0;
    if (!optin[device] &&
        cudaDeviceGetAttribute(&optin[device], cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess)
        return 0;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, lm_head_kernel<ARGMAX, Q4>) != cudaSuccess) return 0;
    // EMBER_HEAD_STAGES caps the depth (a tuning knob; default: all that fit)
    const char *cap = getenv("EMBER_HEAD_STAGES");
    int st = cap && atoi(cap) >= 2 && atoi(cap) < HEAD_MAX_STAGES ? atoi(cap) : HEAD_MAX_STAGES;
    while (st >= 2 && head_smem_bytes(st, stage_bytes, cols) + fa.sharedSizeBytes > (size_t)optin[device]) st--;
    return st >= 2 ? st : 0;
}

template <bool ARGMAX, bool Q4>
static int launch_head_stream(EmberCudaState *s, bool *done) {
    EmberCudaModel *m = s->m;
    const DevMat &w = m->lm_head;
    *done = false;
    const int cols = m->dim, nb = cols / 32;
    if (cols % 32 || nb > 32 || nb < 1) return 0;
    HeadArgs a;
    memset(&a, 0, sizeof(a));
    a.stage_bytes = head_stage_bytes(Q4 ? 1 : 0, cols);
    a.stages = head_stages<ARGMAX, Q4>(m->device, a.stage_bytes, cols);
    if (a.stages == 0) return 0;
    a.q = w.q; a.s = w.s; a.rows = w.rows; a.cols = cols; a.groups = (w.rows + 31) / 32;
    a.x = s->x; a.norm_w = m->final_norm; a.eps = m->eps;
    a.logits = s->logits;
    a.err = s->ctl + CTL_ERR;
    a.part_v = s->am_v; a.part_i = s->am_i; a.ticket = s->am_ticket; a.ctl = s->ctl; a.out = s->out_tokens;
    int grid = s->am_blocks < m->n_sm ? s->am_blocks : m->n_sm;
    if (grid > a.groups) grid = a.groups;
    CK(launch_pdl(lm_head_kernel<ARGMAX, Q4>, grid, HEAD_THREADS, head_smem_bytes(a.stages, a.stage_bytes, cols),
                  s->stream, a));
    *done = true;
    return 0;
}

// final norm + lm_head; with `greedy`, also the argmax and the token / position
// advance when the streaming kernel runs (*fused_tail = true), else the caller
// adds argmax_advance
static int launch_head(EmberCudaState *s, int *count, bool greedy = false, bool *fused_tail = nullptr) {
    EmberCudaModel *m = s->m;
    if (fused_tail) *fused_tail = false;
    const int dt = m->lm_head.dtype;
    if (dt == EMBER_DT_Q8_0 || dt == EMBER_DT_Q4_0) {
        bool done = false;
        const bool q4 = dt == EMBER_DT_Q4_0;
        int rc = greedy ? (q4 ? launch_head_stream<true, true>(s, &done) : launch_head_stream<true, false>(s, &done))
                        : (q4 ? launch_head_stream<false, true>(s, &done) : launch_head_stream<false, false>(s, &done));
        if (rc) return rc;
        if (done) {
            (*count)++;
            if (fused_tail) *fused_tail = greedy;
            return 0;
        }
    }
    GemvArgs a = gemv_base(s);
    a.cols = m->dim;
    a.x = s->x; a.norm_w = m->final_norm; a.eps = m->eps;
    a.seg[0] = seg_of(m->lm_head, s->logits, nullptr);
    a.nseg = 1;
    return run_gemv<IN_NORM, EPI_STORE>(a, m->n_sm, s->stream, count);
}

// The kernels of one token step. with_head: final norm + lm_head; tail: 0 none,
// 1 argmax+advance (greedy), 2 advance (prefill). ids != NULL: prefill feed.
static int record_step(EmberCudaState *s, bool with_layers, bool with_head, int tail, const int *ids, int *count) {
    EmberCudaModel *m = s->m;
    if (with_layers) {
        if (launch_embed(s, ids, count)) return 1;
        for (int l = 0; l < m->n_layers; l++)
            for (int kind = K_QKV; kind <= K_W2; kind++)
                if (launch_layer(s, kind, l, count)) return 1;
    }
    bool fused = false;
    if (with_head && launch_head(s, count, tail == 1, &fused)) return 1;
    if (tail == 1 && !fused) {
        ArgmaxArgs aa;
        aa.logits = s->logits; aa.n = m->vocab; aa.part_v = s->am_v; aa.part_i = s->am_i;
        aa.ticket = s->am_ticket; aa.ctl = s->ctl; aa.out = s->out_tokens;
        CK(launch_pdl(argmax_advance_kernel, s->am_blocks, 256, 0, s->stream, aa));
        (*count)++;
    } else if (tail == 2) {
        CK(launch_pdl(advance_kernel, 1, 32, 0, s->stream, s->ctl));
        (*count)++;
    }
    return 0;
}

// bytes a kernel of one kind must move per launch (weights, activations in and
// out; attention: the cache of positions 0..pos plus this position's writes)
static double mat_bytes(const DevMat &d) {
    double rb = (double)qrow_bytes(d.dtype, d.cols);
    double sb = d.dtype == EMBER_DT_F32 ? 0.0 : (double)(d.cols / 32) * 2.0;
    return (double)d.rows * (rb + sb);
}

static double kernel_bytes(const EmberCudaState *s, int kind, int l, int pos) {
    const EmberCudaModel *m = s->m;
    const int hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
    const double es = s->kv_fp16 ? 2.0 : 4.0;
    const DevLayer &L = m->layers[l];
    switch (kind) {
    case K_QKV: return mat_bytes(L.wq) + mat_bytes(L.wk) + mat_bytes(L.wv) + 8.0 * m->dim + 4.0 * (qd + 2 * kvd);
    case K_ATTN: return 2.0 * kvd * es * (pos + 1) + 4.0 * (qd + 2 * kvd) + qd + qd / 32 * 4.0;
    case K_WO: return mat_bytes(L.wo) + qd + qd / 32 * 4.0 + 8.0 * m->dim;
    case K_W13: return mat_bytes(L.w1) + mat_bytes(L.w3) + 8.0 * m->dim + m->hidden + m->hidden / 32 * 4.0;
    case K_W2: return mat_bytes(L.w2) + m->hidden + m->hidden / 32 * 4.0 + 8.0 * m->dim;
    case K_HEAD: return mat_bytes(m->lm_head) + 8.0 * m->dim + 4.0 * m->vocab;
    }
    return 0.0;
}

static int record_kind(EmberCudaState *s, int kind) {
    cudaStream_t st = s->stream;
    int count = 0;
    if (kind == 0) {
        CK(cudaMemcpyAsync(s->ctl, s->h_ctl, 2 * sizeof(int), cudaMemcpyHostToDevice, st));
        if (record_step(s, true, true, 0, nullptr, &count)) return 1;
        CK(cudaMemcpyAsync(s->h_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(s->h_ctl + CTL_ERR, s->ctl + CTL_ERR, sizeof(int), cudaMemcpyDeviceToHost, st));
        s->launches_per_step = count;
    } else if (kind == 1) {
        if (record_step(s, true, true, 1, nullptr, &count)) return 1;
        s->launches_greedy = count;
    } else if (kind == 2) {
        if (record_step(s, true, false, 2, s->ids, &count)) return 1;
    } else {
        if (record_step(s, false, true, 0, nullptr, &count)) return 1;
        CK(cudaMemcpyAsync(s->h_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, st));
    }
    return 0;
}

// kind 0: forward (ctl from host, logits to host); 1: greedy step;
// 2: prefill step (no head); 3: head only (logits to host)
static int capture(EmberCudaState *s, cudaGraphExec_t *exec, int kind) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    int rc = record_kind(s, kind);
    cudaError_t e = cudaStreamEndCapture(s->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return 1;
    }
    if (e != cudaSuccess) return set_err("graph capture failed: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_err("graph instantiate failed: %s", cudaGetErrorString(e));
    return 0;
}

// a bounded device wait gave up: report it (the step's results are invalid)
static int check_device_error(EmberCudaState *s, int err) {
    if (err == ERR_NONE) return 0;
    cudaMemsetAsync(s->ctl + CTL_ERR, 0, sizeof(int), s->stream);
    cudaStreamSynchronize(s->stream);
    const char *what = err == 11 ? "a hand-off between CTAs of the persistent step never arrived"
                       : err == 12 ? "a weight copy of the persistent step never completed"
                       : err == 13 ? "a cache copy of the persistent step never completed"
                                   : "a bulk copy never completed";
    return set_err("device wait timed out (code %d): %s", err, what);
}

extern "C" int ember_cuda_forward(EmberCudaState *s, int tok, int pos, float *host_logits) {
    CK(cudaSetDevice(s->m->device));
    s->h_ctl[CTL_POS] = pos;
    s->h_ctl[CTL_TOK] = tok;
    s->h_ctl[CTL_ERR] = 0;
    if (s->ps) {
        // one step of the persistent kernel; the logits and the error word back
        CK(cudaMemcpyAsync(s->ctl, s->h_ctl, 2 * sizeof(int), cudaMemcpyHostToDevice, s->stream));
        if (persist_run(s, 1, 0)) return 1;
        CK(cudaMemcpyAsync(s->h_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, s->stream));
        CK(cudaMemcpyAsync(s->h_ctl + CTL_ERR, s->ctl + CTL_ERR, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
    } else {
        if (!s->g_fwd && capture(s, &s->g_fwd, 0)) return 1;
        CK(cudaGraphLaunch(s->g_fwd, s->stream));
    }
    CK(cudaStreamSynchronize(s->stream));
    if (check_device_error(s, s->h_ctl[CTL_ERR])) return 1;
    if (host_logits && host_logits != s->h_logits) memcpy(host_logits, s->h_logits, (size_t)s->m->vocab * 4);
    return 0;
}

static int read_error_word(EmberCudaState *s) {
    int err = 0;
    if (cudaMemcpyAsync(&s->h_ctl[CTL_ERR], s->ctl + CTL_ERR, sizeof(int), cudaMemcpyDeviceToHost, s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess)
        return set_err("reading the device error word failed");
    err = s->h_ctl[CTL_ERR];
    return check_device_error(s, err);
}

// EMBER_PREFILL=steps runs every prefill as single-token steps (for comparisons)
static bool batched_prefill_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("EMBER_PREFILL");
        v = (e && strcmp(e, "steps") == 0) ? 0 : 1;
    }
    return v == 1;
}

static int prefill_impl(EmberCudaState *s, const int *ids, int n, int start, float *host_logits, bool force_batched) {
    CK(cudaSetDevice(s->m->device));
    if (n <= 0) return 0;
    if (force_batched && !(pf_supported(s->m) && pf_fits(s, n, start)))
        return set_err("the batched prefill does not support this model or prompt length");
    if (!s->g_head && capture(s, &s->g_head, 3)) return 1;
    int *hc = s->h_ctl;
    CK(cudaStreamSynchronize(s->stream));
    hc[CTL_POS] = start; hc[CTL_TOK] = 0; hc[CTL_NOUT] = 0; hc[CTL_BASE] = start; hc[CTL_ERR] = 0;
    CK(cudaMemcpyAsync(s->ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->ctl, hc, 5 * sizeof(int), cudaMemcpyHostToDevice, s->stream));
    if (force_batched || (n > 1 && batched_prefill_enabled() && pf_supported(s->m) && pf_fits(s, n, start))) {
        // all layers over the n tokens at once (tensor-core GEMMs), then the head
        if (pf_run_layers(s, s->ids, n, start)) return 1;
    } else {
        if (!s->g_prefill && capture(s, &s->g_prefill, 2)) return 1;
        for (int i = 0; i < n; i++) CK(cudaGraphLaunch(s->g_prefill, s->stream));
    }
    CK(cudaGraphLaunch(s->g_head, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    if (read_error_word(s)) return 1;
    if (host_logits && host_logits != s->h_logits) memcpy(host_logits, s->h_logits, (size_t)s->m->vocab * 4);
    return 0;
}

extern "C" int ember_cuda_prefill(EmberCudaState *s, const int *ids, int n, int start, float *host_logits) {
    return prefill_impl(s, ids, n, start, host_logits, false);
}

int ember_cuda_prefill_batched(EmberCudaState *s, const int *ids, int n, int start, float *host_logits) {
    return prefill_impl(s, ids, n, start, host_logits, true);
}

// the state's greedy-step graph, captured once
int emb::greedy_prepare(EmberCudaState *s) {
    CK(cudaSetDevice(s->m->device));
    return !s->g_greedy && capture(s, &s->g_greedy, 1);
}

// Enqueue n_steps greedy steps on the state's stream without waiting: step i
// feeds t_i at pos + i (t_0 = tok); the chosen tokens go to host_tokens (pinned
// memory, or the copy synchronises) once the steps are done.
int emb::greedy_enqueue(EmberCudaState *s, int tok, int pos, int n_steps, int *host_tokens) {
    if (!s->ps && greedy_prepare(s)) return 1;
    int *hc = s->h_ctl;
    CK(cudaStreamSynchronize(s->stream));
    hc[CTL_POS] = pos; hc[CTL_TOK] = tok; hc[CTL_NOUT] = 0; hc[CTL_BASE] = 0; hc[CTL_ERR] = 0;
    CK(cudaMemcpyAsync(s->ctl, hc, 5 * sizeof(int), cudaMemcpyHostToDevice, s->stream));
    if (s->ps) {
        if (persist_run(s, n_steps, 1)) return 1;   // the whole run in one launch
    } else {
        for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(s->g_greedy, s->stream));
    }
    if (host_tokens) CK(cudaMemcpyAsync(host_tokens, s->out_tokens, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, s->stream));
    return 0;
}

// wait for the state's enqueued work and report a device-side error
int emb::greedy_finish(EmberCudaState *s) {
    CK(cudaSetDevice(s->m->device));
    CK(cudaStreamSynchronize(s->stream));
    return read_error_word(s);
}

extern "C" int ember_cuda_greedy(EmberCudaState *s, int tok, int pos, int n_steps, int *host_tokens,
                                 float *host_logits) {
    CK(cudaSetDevice(s->m->device));
    if (n_steps <= 0) return 0;
    if (greedy_enqueue(s, tok, pos, n_steps, host_tokens)) return 1;
    if (host_logits) CK(cudaMemcpyAsync(host_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, s->stream));
    return greedy_finish(s);
}

extern "C" int ember_cuda_profile_step(EmberCudaState *s, int tok, int pos, float *ms_out, int cap,
                                       int *n_out) {
    CK(cudaSetDevice(s->m->device));
    *n_out = 0;
    std::vector<cudaEvent_t> ev((size_t)cap + 1, nullptr);
    for (auto &e : ev) CK(cudaEventCreate(&e));
    int *hc = s->h_ctl;
    CK(cudaStreamSynchronize(s->stream));
    hc[CTL_POS] = pos; hc[CTL_TOK] = tok; hc[CTL_NOUT] = 0; hc[CTL_BASE] = 0; hc[CTL_ERR] = 0;
    int rc = cudaMemcpyAsync(s->ctl, hc, 5 * sizeof(int), cudaMemcpyHostToDevice, s->stream) != cudaSuccess;
    g_prof_events = ev.data();
    g_prof_n = 0;
    g_prof_cap = cap;
    int count = 0;
    if (!rc) rc = record_step(s, true, true, 1, nullptr, &count);
    const int n = g_prof_n;
    g_prof_events = nullptr;
    if (!rc && cudaEventRecord(ev[n], s->stream) != cudaSuccess) rc = 1;
    if (!rc && cudaStreamSynchronize(s->stream) != cudaSuccess) rc = 1;
    for (int i = 0; i < n && !rc; i++) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, ev[i], ev[i + 1]) != cudaSuccess) rc = 1;
        ms_out[i] = ms;
    }
    for (auto &e : ev) cudaEventDestroy(e);
    if (rc) return set_err("profile step failed: %s", cudaGetErrorString(cudaGetLastError()));
    *n_out = n;
    return read_error_word(s);
}

// ---- timing hooks (CUDA events on the state's stream) ----

static cudaEvent_t g_marks[8];
static int g_marks_ready = 0;

extern "C" int ember_cuda_mark(EmberCudaState *s, int slot) {
    if (slot < 0 || slot >= 8) return set_err("mark slot %d out of range", slot);
    CK(cudaSetDevice(s->m->device));
    if (!g_marks_ready) {
        for (int i = 0; i < 8; i++) CK(cudaEventCreate(&g_marks[i]));
        g_marks_ready = 1;
    }
    CK(cudaEventRecord(g_marks[slot], s->stream));
    return 0;
}

extern "C" int ember_cuda_elapsed_ms(EmberCudaState *s, int a, int b, float *ms) {
    if (!g_marks_ready || a < 0 || a >= 8 || b < 0 || b >= 8) return set_err("bad mark slots");
    CK(cudaSetDevice(s->m->device));
    CK(cudaEventSynchronize(g_marks[b]));
    CK(cudaEventElapsedTime(ms, g_marks[a], g_marks[b]));
    return 0;
}

// Times `reps` rounds of one kernel kind launched for every layer in turn (so
// each launch reads weights that are not in L2), outside any graph, on the
// state's stream between two events. Reports the mean device time per launch
// and the algorithmic bytes per launch (mean over layers, attention at the
// state's current position). The launches change the state's activations and
// cache, so the state is only good for timing afterwards.
extern "C" int ember_cuda_time_kernel(EmberCudaState *s, int kind, int reps, float *ms_per_launch,
                                      double *bytes_per_launch) {
    CK(cudaSetDevice(s->m->device));
    if (kind < K_QKV || kind > K_HEAD || reps <= 0) return set_err("bad kernel kind / reps");
    int hc[CTL_WORDS];
    CK(cudaMemcpy(hc, s->ctl, sizeof(hc), cudaMemcpyDeviceToHost));
    const int L = kind == K_HEAD ? 1 : s->m->n_layers;
    double bytes = 0;
    for (int l = 0; l < L; l++) bytes += kernel_bytes(s, kind, kind == K_HEAD ? 0 : l, hc[CTL_POS]);
    *bytes_per_launch = bytes / L;
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    int count = 0, rc = 0;
    // one untimed round first
    for (int l = 0; l < L && !rc; l++) rc = kind == K_HEAD ? launch_head(s, &count) : launch_layer(s, kind, l, &count);
    if (!rc && cudaEventRecord(e0, s->stream) != cudaSuccess) rc = 1;
    for (int r = 0; r < reps && !rc; r++)
        for (int l = 0; l < L && !rc; l++) rc = kind == K_HEAD ? launch_head(s, &count) : launch_layer(s, kind, l, &count);
    if (!rc && cudaEventRecord(e1, s->stream) != cudaSuccess) rc = 1;
    float ms = 0;
    if (!rc && (cudaEventSynchronize(e1) != cudaSuccess || cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess)) rc = 1;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc) return set_err("kernel timing failed: %s", cudaGetErrorString(cudaGetLastError()));
    *ms_per_launch = ms / (float)(reps * L);
    return read_error_word(s);
}

// ------------------------------------------------------------- op level -------

// ember_matmul / ember_matmul_batch with host pointers: the decode GEMV kernel
// on one input column at a time, device buffers allocated per call.
static int op_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out, int B,
                     BlockQ8_0 *xq) {
    int dev;
    if (pick_device(&dev) || init_kernel_attrs(dev)) return 1;
    if (dtype != EMBER_DT_F32 && dtype != EMBER_DT_Q8_0 && dtype != EMBER_DT_Q4_0)
        return set_err("ember_matmul: dtype %d is not supported", dtype);
    if (dtype != EMBER_DT_F32 && n_in % 32) return set_err("ember_matmul: n_in %% 32 != 0");
    EmberCudaModel tmp;
    tmp.device = dev;
    DevMat dm;
    EmberCudaMat hm = { w, dtype, d_out, n_in };
    int rc = upload_mat(&tmp, &dm, hm);
    float *dx = nullptr, *dout = nullptr, *dxd = nullptr;
    int8_t *dxq = nullptr;
    int *derr = nullptr;
    const int nb = n_in / 32;
    if (!rc) rc = dalloc(&tmp, (void **)&dx, (size_t)n_in * 4) || dalloc(&tmp, (void **)&dout, (size_t)d_out * 4) ||
                  dalloc(&tmp, (void **)&dxq, (size_t)n_in + 16) || dalloc(&tmp, (void **)&dxd, (size_t)nb * 4 + 16) ||
                  dalloc(&tmp, (void **)&derr, 16);
    if (!rc && cudaMemset(derr, 0, 16) != cudaSuccess) rc = set_err("memset");
    std::vector<int8_t> hq(n_in + 16);
    std::vector<float> hd(nb + 1);
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    for (int b = 0; b < B && !rc; b++) {
        if (cudaMemcpy(dx, x + (size_t)b * n_in, (size_t)n_in * 4, cudaMemcpyHostToDevice) != cudaSuccess) { rc = set_err("copy"); break; }
        GemvArgs a;
        memset(&a, 0, sizeof(a));
        a.cols = n_in;
        a.x = dx;
        a.xq_out = dxq;
        a.xd_out = dxd;
        a.err = derr;
        a.seg[0] = seg_of(dm, dout, nullptr);
        a.nseg = 1;
        if (run_gemv<IN_RAW, EPI_STORE>(a, nsm, 0, nullptr)) { rc = 1; break; }
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) { rc = set_err("ember_matmul kernel: %s", cudaGetErrorString(e)); break; }
        int herr = 0;
        if (cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost) != cudaSuccess || herr) { rc = set_err("ember_matmul: device wait timed out"); break; }
        if (cudaMemcpy(out + (size_t)b * d_out, dout, (size_t)d_out * 4, cudaMemcpyDeviceToHost) != cudaSuccess) { rc = set_err("copy"); break; }
        if (dtype != EMBER_DT_F32 && xq) {
            if (cudaMemcpy(hq.data(), dxq, (size_t)n_in, cudaMemcpyDeviceToHost) != cudaSuccess ||
                cudaMemcpy(hd.data(), dxd, (size_t)nb * 4, cudaMemcpyDeviceToHost) != cudaSuccess) { rc = set_err("copy"); break; }
            BlockQ8_0 *blk = xq + (size_t)b * nb;
            for (int j = 0; j < nb; j++) {
                blk[j].d = ember_f32_to_f16(hd[j]);    // hd[j] is an exact fp16 value
                memcpy(blk[j].qs, &hq[(size_t)j * 32], 32);
            }
        }
    }
    model_release(&tmp);
    return rc;
}

extern "C" void ember_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out,
                             BlockQ8_0 *xq) {
    if (op_matmul(out, x, w, dtype, n_in, d_out, 1, xq)) ember_die("cuda: %s", g_err);
}

// quantized weights, two or more columns: the tensor-core GEMM of the batched
// prefill (ref src/kernels.c:227-264); otherwise one GEMV per column
static int op_matmul_batch(float *out, const float *x, const void *w, int dtype, int n_in, int d_out, int B,
                           BlockQ8_0 *xq) {
    int dev;
    if (pick_device(&dev)) return 1;
    if (n_in % 32) return set_err("ember_matmul_batch: n_in %% 32 != 0");
    EmberCudaModel tmp;
    tmp.device = dev;
    DevMat dm;
    EmberCudaMat hm = { w, dtype, d_out, n_in };
    int rc = upload_mat(&tmp, &dm, hm);
    if (!rc) rc = pf_matmul_batch(dev, out, x, dm, B, xq);
    model_release(&tmp);
    return rc;
}

extern "C" void ember_matmul_batch(float *out, const float *x, const void *w, int dtype, int n_in, int d_out,
                                   int B, BlockQ8_0 *xq) {
    if (B <= 0) return;
    const bool gemm = B > 1 && (dtype == EMBER_DT_Q8_0 || dtype == EMBER_DT_Q4_0) && batched_prefill_enabled();
    if (gemm ? op_matmul_batch(out, x, w, dtype, n_in, d_out, B, xq) : op_matmul(out, x, w, dtype, n_in, d_out, B, xq))
        ember_die("cuda: %s", g_err);
}

#ifdef EMBER_PROBES
// profiling build only: phase probes and per-launch wait times
extern "C" int ember_cuda_probe_read(unsigned long long *phases, unsigned long long *waits, unsigned *count, int reset) {
    if (cudaDeviceSynchronize() != cudaSuccess) return 1;
    if (cudaMemcpyFromSymbol(phases, g_probe, sizeof(g_probe)) != cudaSuccess) return 1;
    if (cudaMemcpyFromSymbol(count, g_wait_count, sizeof(unsigned)) != cudaSuccess) return 1;
    if (cudaMemcpyFromSymbol(waits, g_wait_times, sizeof(g_wait_times)) != cudaSuccess) return 1;
    if (reset) {
        unsigned z = 0;
        if (cudaMemcpyToSymbol(g_wait_count, &z, sizeof(z)) != cudaSuccess) return 1;
    }
    return 0;
}
#endif
