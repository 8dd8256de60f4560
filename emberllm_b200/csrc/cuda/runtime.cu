// runtime.cu — the ember_cuda_* shim: device weights, run states, the captured
// token-step graphs, and the op-level ember_matmul entry points.
//
// Device layout. A .ember Q8_0 row is an array of 34-byte {fp16 d; int8 qs[32]}
// blocks (18-byte for Q4_0), so rows are not 16-byte aligned and scales sit
// between the quants. At upload every quantized matrix is split into a
// row-major byte array (32 or 16 bytes per block, every row and block 16-byte
// aligned, so a warp streams a tile of consecutive rows with 128-bit loads) and
// a separate [rows][cols/32] fp16 scale array. The KV cache is laid out per
// layer as [n_kv][ctx][head_dim] so one head's keys for consecutive positions
// are contiguous.
//
// Execution. One token step is a fixed sequence of kernels (kernels.cuh) that
// read the position and token from device memory, captured once per state into
// CUDA graphs and replayed for every token. Kernels are launched with
// programmatic stream serialization so each one starts while its predecessor
// finishes and prefetches its own weights into L2 before waiting on the data it
// needs.
#include <cuda_runtime.h>

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "ember_cuda.h"
#include "ember_ops.h"
#include "kernels.cuh"

using namespace emb;

// ------------------------------------------------------------------ errors ----

static char g_err[512] = "no error";

static int set_err(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return 1;
}

#define CK(call)                                                                           \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return set_err("%s (%s:%d: %s)", cudaGetErrorString(e_), __FILE__, __LINE__, #call); \
    } while (0)

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

// ------------------------------------------------------------------ model -----

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

struct EmberCudaModel {
    int device = 0, n_sm = 148;
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, vocab, qk_norm, rope_neox;
    float eps;
    DevMat tok_emb, lm_head;
    float *final_norm = nullptr;
    std::vector<DevLayer> layers;
    ExpfDev ex;
    std::vector<void *> allocs;
    uint64_t bytes = 0;
};

static int dalloc(EmberCudaModel *m, void **p, size_t n) {
    CK(cudaMalloc(p, n ? n : 16));
    m->allocs.push_back(*p);
    m->bytes += n;
    return 0;
}

static int upload_vec(EmberCudaModel *m, float **dst, const float *src, int n) {
    if (!src) { *dst = nullptr; return 0; }
    if (dalloc(m, (void **)dst, (size_t)n * 4)) return 1;
    CK(cudaMemcpy(*dst, src, (size_t)n * 4, cudaMemcpyHostToDevice));
    return 0;
}

// Split AoS blocks into quant rows + scale rows and upload.
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
    if (dalloc(m, (void **)&d->q, qn) || dalloc(m, (void **)&d->s, sn)) return 1;
    // repack in row chunks to bound the host staging buffer
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
        m->ex.p = *e;
        uint32_t *slots = nullptr;
        rc = dalloc(m, (void **)&slots, (size_t)e->n_slots * 8);
        if (!rc && cudaMemcpy(slots, e->slots, (size_t)e->n_slots * 8, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = set_err("expf table upload failed");
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

struct EmberCudaState {
    EmberCudaModel *m = nullptr;
    int ctx = 0, kv_fp16 = 0;
    cudaStream_t stream = nullptr;
    std::vector<void *> allocs;
    // device buffers
    float *x, *q, *k, *v, *att, *od, *of, *hd, *hf, *logits;
    int8_t *oq, *hq;
    void *kc, *vc;
    float2 *rope;
    int *ctl, *ids, *out_tokens;
    float *am_v;
    int *am_i;
    unsigned *am_ticket;
    int am_blocks;
    // pinned host
    float *h_logits = nullptr;
    int *h_ctl = nullptr;
    // graphs
    cudaGraphExec_t g_fwd = nullptr, g_greedy = nullptr, g_prefill = nullptr, g_head = nullptr;
    int launches_per_step = 0;
};

static int init_kernel_attrs(int device);

static int salloc(EmberCudaState *s, void **p, size_t n) {
    CK(cudaMalloc(p, n ? n : 16));
    s->allocs.push_back(*p);
    return 0;
}

static void state_release(EmberCudaState *s) {
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
    const int hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
    const size_t es = kv_fp16 ? 2 : 4;
    const size_t kv_bytes = (size_t)m->n_layers * ctx * kvd * es;
    s->am_blocks = m->n_sm;
    int rc = 0;
    rc |= salloc(s, (void **)&s->x, (size_t)m->dim * 4);
    rc |= salloc(s, (void **)&s->q, (size_t)qd * 4);
    rc |= salloc(s, (void **)&s->k, (size_t)kvd * 4);
    rc |= salloc(s, (void **)&s->v, (size_t)kvd * 4);
    rc |= salloc(s, (void **)&s->att, (size_t)m->n_heads * ctx * 4);
    rc |= salloc(s, (void **)&s->oq, (size_t)qd);
    rc |= salloc(s, (void **)&s->od, (size_t)qd / 32 * 4 + 4);
    rc |= salloc(s, (void **)&s->of, (size_t)qd * 4);
    rc |= salloc(s, (void **)&s->hq, (size_t)m->hidden + 16);
    rc |= salloc(s, (void **)&s->hd, (size_t)m->hidden / 32 * 4 + 4);
    rc |= salloc(s, (void **)&s->hf, (size_t)m->hidden * 4);
    rc |= salloc(s, (void **)&s->logits, (size_t)m->vocab * 4);
    rc |= salloc(s, &s->kc, kv_bytes);
    rc |= salloc(s, &s->vc, kv_bytes);
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
        cudaMemset(s->kc, 0, kv_bytes) != cudaSuccess || cudaMemset(s->vc, 0, kv_bytes) != cudaSuccess ||
        cudaMemset(s->ctl, 0, CTL_WORDS * 4) != cudaSuccess || cudaMemset(s->am_ticket, 0, 4) != cudaSuccess ||
        cudaMemset(s->logits, 0, (size_t)m->vocab * 4) != cudaSuccess) {
        set_err("state initialisation failed: %s", cudaGetErrorString(cudaGetLastError()));
        state_release(s);
        delete s;
        return 1;
    }
    memset(s->h_logits, 0, (size_t)m->vocab * 4);
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

// ------------------------------------------------------------------ launches --

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Raise the dynamic shared-memory limit of every gemv instantiation once per
// device, outside any stream capture.
static int init_kernel_attrs(int device) {
    static int done_mask = 0;
    if (device < 31 && (done_mask >> device) & 1) return 0;
    const int lim = 200 * 1024;
    CK(cudaFuncSetAttribute(gemv_kernel<IN_RAW, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
    CK(cudaFuncSetAttribute(gemv_kernel<IN_NORM, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
    CK(cudaFuncSetAttribute(gemv_kernel<IN_NORM, EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
    CK(cudaFuncSetAttribute(gemv_kernel<IN_QUANT, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
    if (device < 31) done_mask |= 1 << device;
    return 0;
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

static void gemv_tiles(GemvArgs &a) {
    a.tiles[0] = 0;
    for (int k = 0; k < a.nseg; k++) a.tiles[k + 1] = a.tiles[k] + (a.seg[k].rows + GEMV_ROWS - 1) / GEMV_ROWS;
    for (int k = a.nseg + 1; k < 4; k++) a.tiles[k] = a.tiles[a.nseg];
}

template <int IN, int EPI>
static cudaError_t run_gemv(GemvArgs a, int n_sm, cudaStream_t st, int *count) {
    if (EPI == EPI_SWIGLU) {
        a.tiles[0] = 0;
        a.tiles[1] = a.tiles[2] = a.tiles[3] = (a.seg[0].rows + GEMV_ROWS - 1) / GEMV_ROWS;
        a.nseg = 1;   // tiles[nseg] is the pair count; both segments are read per tile
    } else {
        gemv_tiles(a);
    }
    const int total = a.tiles[a.nseg];
    int grid = total < 2 * n_sm ? total : 2 * n_sm;
    if (grid < 1) grid = 1;
    const int per_cta = (total + grid - 1) / grid;
    a.prefetch_tiles = per_cta < 4 ? per_cta : 4;
    bool f32 = false;
    for (int k = 0; k < (EPI == EPI_SWIGLU ? 2 : a.nseg); k++) f32 |= a.seg[k].dtype == EMBER_DT_F32;
    const size_t smem = gemv_smem_bytes(a.cols, IN != IN_QUANT || f32);
    if (count) (*count)++;
    return launch_pdl(gemv_kernel<IN, EPI>, grid, GEMV_THREADS, smem, st, a);
}

// The kernels of one token step. with_head: final norm + lm_head; tail: 0 none,
// 1 argmax+advance (greedy), 2 advance (prefill). ids != NULL: prefill feed.
static int record_step(EmberCudaState *s, bool with_layers, bool with_head, int tail, const int *ids, int *count) {
    EmberCudaModel *m = s->m;
    cudaStream_t st = s->stream;
    const int hd = m->head_dim, kvd = m->n_kv * hd;
    const size_t es = s->kv_fp16 ? 2 : 4;
    if (with_layers) {
        EmbedArgs ea;
        ea.q = m->tok_emb.q; ea.s = m->tok_emb.s; ea.dtype = m->tok_emb.dtype; ea.dim = m->dim;
        ea.ctl = s->ctl; ea.ids = ids; ea.x = s->x;
        CK(launch_pdl(embed_kernel, 1, 256, 0, st, ea));
        (*count)++;
        for (int l = 0; l < m->n_layers; l++) {
            const DevLayer &L = m->layers[l];
            GemvArgs a;
            memset(&a, 0, sizeof(a));
            a.ex = m->ex;
            a.cols = m->dim;
            a.x = s->x; a.norm_w = L.attn_norm; a.eps = m->eps;
            a.seg[0] = seg_of(L.wq, s->q, L.bq);
            a.seg[1] = seg_of(L.wk, s->k, L.bk);
            a.seg[2] = seg_of(L.wv, s->v, L.bv);
            a.nseg = 3;
            CK((run_gemv<IN_NORM, EPI_STORE>(a, m->n_sm, st, count)));

            AttnArgs at;
            at.q = s->q; at.k = s->k; at.v = s->v;
            at.kc = (char *)s->kc + (size_t)l * s->ctx * kvd * es;
            at.vc = (char *)s->vc + (size_t)l * s->ctx * kvd * es;
            at.q_norm = L.q_norm; at.k_norm = L.k_norm;
            at.rope = s->rope; at.ctl = s->ctl; at.att = s->att;
            at.oq = s->oq; at.od = s->od; at.of = s->of;
            at.nh = m->n_heads; at.nkv = m->n_kv; at.hd = hd; at.ctx = s->ctx;
            at.neox = m->rope_neox; at.eps = m->eps; at.ex = m->ex;
            if (s->kv_fp16) CK(launch_pdl(attn_decode_kernel<__half>, m->n_heads, ATTN_THREADS, 0, st, at));
            else CK(launch_pdl(attn_decode_kernel<float>, m->n_heads, ATTN_THREADS, 0, st, at));
            (*count)++;

            memset(&a, 0, sizeof(a));
            a.ex = m->ex;
            a.cols = m->n_heads * hd;
            a.xq = s->oq; a.xd = s->od; a.xf = s->of;
            a.seg[0] = seg_of(L.wo, s->x, nullptr);
            a.nseg = 1;
            CK((run_gemv<IN_QUANT, EPI_RESID>(a, m->n_sm, st, count)));

            memset(&a, 0, sizeof(a));
            a.ex = m->ex;
            a.cols = m->dim;
            a.x = s->x; a.norm_w = L.ffn_norm; a.eps = m->eps;
            a.seg[0] = seg_of(L.w1, nullptr, nullptr);
            a.seg[1] = seg_of(L.w3, nullptr, nullptr);
            a.nseg = 2;
            a.hq = s->hq; a.hd = s->hd; a.hf = s->hf;
            CK((run_gemv<IN_NORM, EPI_SWIGLU>(a, m->n_sm, st, count)));

            memset(&a, 0, sizeof(a));
            a.ex = m->ex;
            a.cols = m->hidden;
            a.xq = s->hq; a.xd = s->hd; a.xf = s->hf;
            a.seg[0] = seg_of(L.w2, s->x, nullptr);
            a.nseg = 1;
            CK((run_gemv<IN_QUANT, EPI_RESID>(a, m->n_sm, st, count)));
        }
    }
    if (with_head) {
        GemvArgs a;
        memset(&a, 0, sizeof(a));
        a.ex = m->ex;
        a.cols = m->dim;
        a.x = s->x; a.norm_w = m->final_norm; a.eps = m->eps;
        a.seg[0] = seg_of(m->lm_head, s->logits, nullptr);
        a.nseg = 1;
        CK((run_gemv<IN_NORM, EPI_STORE>(a, m->n_sm, st, count)));
    }
    if (tail == 1) {
        ArgmaxArgs aa;
        aa.logits = s->logits; aa.n = m->vocab; aa.part_v = s->am_v; aa.part_i = s->am_i;
        aa.ticket = s->am_ticket; aa.ctl = s->ctl; aa.out = s->out_tokens;
        CK(launch_pdl(argmax_advance_kernel, s->am_blocks, 256, 0, st, aa));
        (*count)++;
    } else if (tail == 2) {
        CK(launch_pdl(advance_kernel, 1, 32, 0, st, s->ctl));
        (*count)++;
    }
    return 0;
}

static int record_kind(EmberCudaState *s, int kind) {
    cudaStream_t st = s->stream;
    int count = 0;
    if (kind == 0) {
        CK(cudaMemcpyAsync(s->ctl, s->h_ctl, 2 * sizeof(int), cudaMemcpyHostToDevice, st));
        if (record_step(s, true, true, 0, nullptr, &count)) return 1;
        CK(cudaMemcpyAsync(s->h_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, st));
        s->launches_per_step = count;
    } else if (kind == 1) {
        if (record_step(s, true, true, 1, nullptr, &count)) return 1;
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

extern "C" int ember_cuda_forward(EmberCudaState *s, int tok, int pos, float *host_logits) {
    CK(cudaSetDevice(s->m->device));
    if (!s->g_fwd && capture(s, &s->g_fwd, 0)) return 1;
    s->h_ctl[CTL_POS] = pos;
    s->h_ctl[CTL_TOK] = tok;
    CK(cudaGraphLaunch(s->g_fwd, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    if (host_logits && host_logits != s->h_logits) memcpy(host_logits, s->h_logits, (size_t)s->m->vocab * 4);
    return 0;
}

extern "C" int ember_cuda_prefill(EmberCudaState *s, const int *ids, int n, int start, float *host_logits) {
    CK(cudaSetDevice(s->m->device));
    if (n <= 0) return 0;
    if (!s->g_prefill && capture(s, &s->g_prefill, 2)) return 1;
    if (!s->g_head && capture(s, &s->g_head, 3)) return 1;
    int ctl[CTL_WORDS] = { start, 0, 0, start };
    CK(cudaMemcpyAsync(s->ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice, s->stream));
    for (int i = 0; i < n; i++) CK(cudaGraphLaunch(s->g_prefill, s->stream));
    CK(cudaGraphLaunch(s->g_head, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    if (host_logits && host_logits != s->h_logits) memcpy(host_logits, s->h_logits, (size_t)s->m->vocab * 4);
    return 0;
}

extern "C" int ember_cuda_greedy(EmberCudaState *s, int tok, int pos, int n_steps, int *host_tokens,
                                 float *host_logits) {
    CK(cudaSetDevice(s->m->device));
    if (n_steps <= 0) return 0;
    if (!s->g_greedy && capture(s, &s->g_greedy, 1)) return 1;
    int ctl[CTL_WORDS] = { pos, tok, 0, 0 };
    CK(cudaMemcpyAsync(s->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice, s->stream));
    for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(s->g_greedy, s->stream));
    if (host_tokens) CK(cudaMemcpyAsync(host_tokens, s->out_tokens, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, s->stream));
    if (host_logits) CK(cudaMemcpyAsync(host_logits, s->logits, (size_t)s->m->vocab * 4, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    return 0;
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
    const int nb = n_in / 32;
    if (!rc) rc = dalloc(&tmp, (void **)&dx, (size_t)n_in * 4) || dalloc(&tmp, (void **)&dout, (size_t)d_out * 4) ||
                  dalloc(&tmp, (void **)&dxq, (size_t)n_in + 16) || dalloc(&tmp, (void **)&dxd, (size_t)nb * 4 + 4);
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
        a.seg[0] = seg_of(dm, dout, nullptr);
        a.nseg = 1;
        cudaError_t e = run_gemv<IN_RAW, EPI_STORE>(a, nsm, 0, nullptr);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) { rc = set_err("ember_matmul kernel: %s", cudaGetErrorString(e)); break; }
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

extern "C" void ember_matmul_batch(float *out, const float *x, const void *w, int dtype, int n_in, int d_out,
                                   int B, BlockQ8_0 *xq) {
    if (B <= 0) return;
    if (op_matmul(out, x, w, dtype, n_in, d_out, B, xq)) ember_die("cuda: %s", g_err);
}
