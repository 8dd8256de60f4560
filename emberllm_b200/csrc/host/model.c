/* model.c — run states and the token-loop entry points (replaces ref
 * src/model.c:116-414).
 *
 * The host side keeps the reference's contract: tensor resolution by name with
 * the same fatal messages (ref src/model.c:144-171), range checks on token ids
 * and positions (ref src/model.c:306-307, :368-371), and a logits buffer owned by
 * the state and returned by every call. The arithmetic runs on the GPU through
 * the ember_cuda_* shim; the host contributes the two tables whose values come
 * from this host's C math library (RoPE cos/sin and the expf exception list), so
 * that the device reproduces the reference's results bit for bit.
 */
#include "model_internal.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct EmberState {
    const EmberModel *m;
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, kv_dim, vocab, ctx, kv_fp16;
    EmberCudaState *dev;
    float *logits;          /* pinned host buffer owned by dev */
};

static void cuda_check(int rc, const char *what) {
    if (rc != 0) ember_die("cuda: %s: %s", what, ember_cuda_error());
}

/* Look a tensor up by a printf-style name (ref src/model.c:102-110). */
static const EmberTensor *find(const EmberModel *m, const char *fmt, int layer) {
    char name[48];
    if (layer >= 0) snprintf(name, sizeof(name), fmt, layer);
    else snprintf(name, sizeof(name), "%s", fmt);
    return ember_model_tensor(m, name);
}

static size_t row_bytes(int dtype, int cols) {
    switch (dtype) {
    case EMBER_DT_F32: return (size_t)cols * 4;
    case EMBER_DT_Q8_0: return (size_t)(cols / EMBER_Q_BLOCK) * sizeof(BlockQ8_0);
    case EMBER_DT_Q4_0: return (size_t)(cols / EMBER_Q_BLOCK) * sizeof(BlockQ4_0);
    default: return 0;
    }
}

/* Resolve a weight matrix [rows, cols]; NULL data when absent. Shapes come from
 * the header, as in the reference; the stored size is checked against them so a
 * truncated table entry dies here instead of reading past the mapping. */
static EmberCudaMat mat(const EmberModel *m, const char *fmt, int layer, int rows, int cols) {
    EmberCudaMat w = { NULL, EMBER_DT_F32, rows, cols };
    const EmberTensor *t = find(m, fmt, layer);
    if (!t) return w;
    const void *p = ember_model_data(m, t);
    if (!p) return w;
    if (t->dtype != EMBER_DT_F32 && t->dtype != EMBER_DT_Q8_0 && t->dtype != EMBER_DT_Q4_0)
        ember_die("tensor '%.48s' has dtype %d, which this backend does not run", t->name, t->dtype);
    if (t->dtype != EMBER_DT_F32 && cols % EMBER_Q_BLOCK != 0)
        ember_die("tensor '%.48s' is quantized but its rows are not whole blocks", t->name);
    if ((uint64_t)rows * row_bytes(t->dtype, cols) > t->nbytes)
        ember_die("tensor '%.48s' is smaller than its [%d, %d] shape", t->name, rows, cols);
    w.data = p;
    w.dtype = t->dtype;
    return w;
}

static const float *vec(const EmberModel *m, const char *fmt, int layer, int n) {
    const EmberTensor *t = find(m, fmt, layer);
    if (!t) return NULL;
    const void *p = ember_model_data(m, t);
    if (!p) return NULL;
    if (t->dtype != EMBER_DT_F32 || t->nbytes < (uint64_t)n * 4)
        ember_die("tensor '%.48s' must hold %d fp32 values", t->name, n);
    return (const float *)p;
}

/* Upload the model the first time a state needs it. */
static void ensure_uploaded(EmberModel *m) {
    if (m->dev) return;
    const EmberHeader *h = m->hdr;
    int L = h->n_layers, dim = h->dim, hidden = h->hidden_dim, hd = h->head_dim;
    int qd = h->n_heads * hd, kvd = h->n_kv_heads * hd;

    EmberCudaModelDesc d;
    memset(&d, 0, sizeof(d));
    d.dim = dim; d.hidden = hidden; d.n_layers = L; d.n_heads = h->n_heads;
    d.n_kv_heads = h->n_kv_heads; d.head_dim = hd; d.vocab = h->vocab_size;
    d.norm_eps = h->norm_eps;
    d.qk_norm = (h->flags & EMBER_FLAG_QK_NORM) != 0;
    d.rope_neox = h->rope_style == EMBER_ROPE_NEOX;

    EmberCudaMat *mats = ember_xcalloc((size_t)7 * L, sizeof(EmberCudaMat), "layer weights");
    const float **vecs = ember_xcalloc((size_t)9 * L, sizeof(float *), "layer vectors");
    EmberCudaMat *wq = mats, *wk = mats + L, *wv = mats + 2 * L, *wo = mats + 3 * L;
    EmberCudaMat *w1 = mats + 4 * L, *w2 = mats + 5 * L, *w3 = mats + 6 * L;
    const float **an = vecs, **fn = vecs + L, **qn = vecs + 2 * L, **kn = vecs + 3 * L;
    const float **bq = vecs + 4 * L, **bk = vecs + 5 * L, **bv = vecs + 6 * L;

    for (int l = 0; l < L; l++) {
        wq[l] = mat(m, "layers.%d.wq", l, qd, dim);
        wk[l] = mat(m, "layers.%d.wk", l, kvd, dim);
        wv[l] = mat(m, "layers.%d.wv", l, kvd, dim);
        wo[l] = mat(m, "layers.%d.wo", l, dim, qd);
        w1[l] = mat(m, "layers.%d.w1", l, hidden, dim);
        w2[l] = mat(m, "layers.%d.w2", l, dim, hidden);
        w3[l] = mat(m, "layers.%d.w3", l, hidden, dim);
        an[l] = vec(m, "layers.%d.attn_norm", l, dim);
        fn[l] = vec(m, "layers.%d.ffn_norm", l, dim);
        qn[l] = vec(m, "layers.%d.q_norm", l, hd);
        kn[l] = vec(m, "layers.%d.k_norm", l, hd);
        bq[l] = vec(m, "layers.%d.wq_bias", l, qd);
        bk[l] = vec(m, "layers.%d.wk_bias", l, kvd);
        bv[l] = vec(m, "layers.%d.wv_bias", l, kvd);
    }
    d.tok_emb = mat(m, "tok_embeddings", -1, h->vocab_size, dim);
    d.final_norm = vec(m, "final_norm", -1, dim);
    d.lm_head = (h->flags & EMBER_FLAG_TIED_EMBED) ? d.tok_emb
                                                    : mat(m, "lm_head", -1, h->vocab_size, dim);
    /* the reference's existence checks and messages (ref src/model.c:163-171) */
    if (!d.tok_emb.data) ember_die("model is missing tensor 'tok_embeddings'");
    if (!d.final_norm) ember_die("model is missing tensor 'final_norm'");
    if (!d.lm_head.data) ember_die("model is missing tensor 'lm_head' (and is not tied)");
    for (int l = 0; l < L; l++) {
        if (!wq[l].data || !wk[l].data || !wv[l].data || !wo[l].data || !w1[l].data ||
            !w2[l].data || !w3[l].data || !an[l] || !fn[l])
            ember_die("model is missing a required tensor in layer %d", l);
        /* the reference applies QK-norm only where q_norm exists (ref src/model.c:386) */
        if (d.qk_norm && qn[l] && !kn[l])
            ember_die("model has layers.%d.q_norm but no layers.%d.k_norm", l, l);
        if (!d.qk_norm) { qn[l] = NULL; kn[l] = NULL; }
        if (!qn[l]) kn[l] = NULL;
    }
    if (d.tok_emb.dtype == EMBER_DT_Q4_0)
        ember_die("a Q4_0 token-embedding table is not supported (emberllm keeps it at Q8_0)");

    d.wq = wq; d.wk = wk; d.wv = wv; d.wo = wo; d.w1 = w1; d.w2 = w2; d.w3 = w3;
    d.attn_norm = an; d.ffn_norm = fn; d.q_norm = qn; d.k_norm = kn;
    d.b_q = bq; d.b_k = bk; d.b_v = bv;

    EmberExpfParams ex;
    if (ember_host_expf_params(&ex) != 0) ember_die("could not build the expf table");
    cuda_check(ember_cuda_model_upload(&d, &ex, &m->dev), "model upload");
    free(mats);
    free(vecs);
}

EmberState *ember_state_new(const EmberModel *m, int ctx_len) {
    return ember_state_new_ex(m, ctx_len, 0);
}

EmberState *ember_state_new_ex(const EmberModel *m, int ctx_len, int kv_fp16) {
    const EmberHeader *h = ember_model_header(m);
    if (h->n_heads <= 0 || h->n_kv_heads <= 0 || h->n_heads % h->n_kv_heads != 0)
        ember_die("n_heads (%d) must be a positive multiple of n_kv_heads (%d)", h->n_heads,
                  h->n_kv_heads);
    if (h->head_dim <= 0 || h->head_dim % EMBER_Q_BLOCK != 0 || h->head_dim > 256)
        ember_die("head_dim %d is not supported (multiples of 32 up to 256)", h->head_dim);
    if (h->hidden_dim <= 0 || h->max_seq_len <= 0)
        ember_die("header has non-positive hidden_dim or max_seq_len");
    ensure_uploaded((EmberModel *)m);

    EmberState *s = ember_xcalloc(1, sizeof(*s), "EmberState");
    s->m = m;
    s->dim = h->dim; s->hidden = h->hidden_dim; s->n_layers = h->n_layers;
    s->n_heads = h->n_heads; s->n_kv = h->n_kv_heads; s->head_dim = h->head_dim;
    s->kv_dim = h->n_kv_heads * h->head_dim; s->vocab = h->vocab_size;
    s->kv_fp16 = kv_fp16 ? 1 : 0;
    s->ctx = (ctx_len > 0 && ctx_len < h->max_seq_len) ? ctx_len : h->max_seq_len;

    size_t n_rope = (size_t)s->ctx * (size_t)(s->head_dim / 2) * 2;
    float *rope = ember_xmalloc(n_rope * sizeof(float), "rope table");
    ember_host_rope_table(rope, s->ctx, s->head_dim, h->rope_theta);
    cuda_check(ember_cuda_state_new(m->dev, s->ctx, s->kv_fp16, rope, &s->dev), "state");
    free(rope);
    s->logits = ember_cuda_state_host_logits(s->dev);
    return s;
}

void ember_state_free(EmberState *s) {
    if (!s) return;
    ember_cuda_state_free(s->dev);
    free(s);
}

float *ember_forward(EmberModel *m, EmberState *s, int tok, int pos) {
    (void)m;
    if (tok < 0 || tok >= s->vocab) ember_die("token id %d out of range [0,%d)", tok, s->vocab);
    if (pos < 0 || pos >= s->ctx) ember_die("position %d out of range [0,%d)", pos, s->ctx);
    cuda_check(ember_cuda_forward(s->dev, tok, pos, s->logits), "forward");
    return s->logits;
}

float *ember_prefill(EmberModel *m, EmberState *s, const int *ids, int n, int start) {
    (void)m;
    if (n <= 0) return s->logits;
    for (int b = 0; b < n; b++)
        if (ids[b] < 0 || ids[b] >= s->vocab)
            ember_die("token id %d out of range [0,%d)", ids[b], s->vocab);
    if (start < 0 || start > s->ctx - n)
        ember_die("prefill of %d tokens at position %d does not fit the context of %d", n, start,
                  s->ctx);
    cuda_check(ember_cuda_prefill(s->dev, ids, n, start, s->logits), "prefill");
    return s->logits;
}

float *ember_forward_greedy(EmberModel *m, EmberState *s, int tok, int pos, int n,
                            int *out_tokens) {
    (void)m;
    if (n <= 0) return s->logits;
    if (tok < 0 || tok >= s->vocab) ember_die("token id %d out of range [0,%d)", tok, s->vocab);
    if (pos < 0 || pos > s->ctx - n)
        ember_die("%d greedy steps from position %d do not fit the context of %d", n, pos, s->ctx);
    cuda_check(ember_cuda_greedy(s->dev, tok, pos, n, out_tokens, s->logits), "greedy");
    return s->logits;
}

EmberCudaState *ember_state_cuda(EmberState *s) { return s->dev; }

/* ---- sampling on the device (extension) ----
 * The sampler's random stream is xorshift64* (Vigna's generator: shifts 12, 25,
 * 27, multiplier 0x2545F4914F6CDD1D, high 32 bits), mapped to [0, 1) as the top 24
 * bits / 2^24, the draw the reference's sampler makes (ref src/sample.c:98-105);
 * its steps must match for a seed to reproduce the reference's tokens. */
static uint32_t xs64_u32(uint64_t *state) {
    uint64_t x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return (uint32_t)((x * 0x2545F4914F6CDD1DULL) >> 32);
}

int ember_sample_device(EmberState *s, const EmberSampleParams *p, uint64_t *rng_state, const int *history,
                        int hist_len) {
    if (!p || !rng_state) ember_die("ember_sample_device: null sampler settings");
    /* the reference draws once, after the softmax, only when temperature > 0 */
    float u = 0.0f;
    if (p->temperature > 0.0f) u = (float)(xs64_u32(rng_state) >> 8) / 16777216.0f;
    int tok = 0;
    cuda_check(ember_cuda_sample(s->dev, p, u, history, history ? hist_len : 0, &tok), "sample");
    return tok;
}

/* ---- batched greedy decode of independent streams (extension) ---- */
struct EmberBatch {
    EmberCudaBatch *dev;
    int n_streams, ctx, vocab;
    float *logits;            /* [vocab]: the last prompt's logits */
};

EmberBatch *ember_batch_new(EmberModel *m, int n_streams, int ctx_len, int kv_fp16, int max_steps) {
    const EmberHeader *h = ember_model_header(m);
    if (h->n_heads <= 0 || h->n_kv_heads <= 0 || h->n_heads % h->n_kv_heads != 0)
        ember_die("n_heads (%d) must be a positive multiple of n_kv_heads (%d)", h->n_heads, h->n_kv_heads);
    if (h->head_dim <= 0 || h->head_dim % EMBER_Q_BLOCK != 0 || h->head_dim > 256)
        ember_die("head_dim %d is not supported (multiples of 32 up to 256)", h->head_dim);
    ensure_uploaded(m);
    EmberBatch *b = ember_xcalloc(1, sizeof(*b), "EmberBatch");
    b->n_streams = n_streams;
    b->vocab = h->vocab_size;
    b->ctx = (ctx_len > 0 && ctx_len < h->max_seq_len) ? ctx_len : h->max_seq_len;
    size_t n_rope = (size_t)b->ctx * (size_t)(h->head_dim / 2) * 2;
    float *rope = ember_xmalloc(n_rope * sizeof(float), "rope table");
    ember_host_rope_table(rope, b->ctx, h->head_dim, h->rope_theta);
    cuda_check(ember_cuda_batch_new(m->dev, n_streams, b->ctx, kv_fp16 ? 1 : 0, rope, max_steps, &b->dev),
               "batch");
    free(rope);
    b->logits = ember_xmalloc((size_t)b->vocab * sizeof(float), "batch logits");
    return b;
}

void ember_batch_free(EmberBatch *b) {
    if (!b) return;
    ember_cuda_batch_free(b->dev);
    free(b->logits);
    free(b);
}

EmberCudaBatch *ember_batch_cuda(EmberBatch *b) { return b ? b->dev : NULL; }

float *ember_batch_prefill(EmberBatch *b, int stream, const int *ids, int n) {
    if (stream < 0 || stream >= b->n_streams) ember_die("stream %d out of range [0,%d)", stream, b->n_streams);
    if (n <= 0 || n > b->ctx) ember_die("prompt of %d tokens does not fit the context of %d", n, b->ctx);
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= b->vocab) ember_die("token id %d out of range [0,%d)", ids[i], b->vocab);
    cuda_check(ember_cuda_batch_prefill(b->dev, stream, ids, n, b->logits), "batch prefill");
    return b->logits;
}

void ember_batch_greedy(EmberBatch *b, const int *toks, const int *pos, int n_steps, int *out_tokens,
                        float *out_logits) {
    for (int i = 0; i < b->n_streams; i++) {
        if (toks[i] < 0 || toks[i] >= b->vocab) ember_die("token id %d out of range [0,%d)", toks[i], b->vocab);
        if (pos[i] < 0 || pos[i] + n_steps > b->ctx)
            ember_die("stream %d: %d steps from position %d do not fit the context of %d", i, n_steps, pos[i],
                      b->ctx);
    }
    cuda_check(ember_cuda_batch_greedy(b->dev, toks, pos, n_steps, out_tokens, out_logits), "batch greedy");
}
