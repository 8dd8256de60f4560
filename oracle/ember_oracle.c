/* ember_oracle.c — TEST INFRASTRUCTURE ONLY: a CPU restatement of emberllm's
 * token loop, used to check the GPU library. The product never links or calls it.
 *
 * Each function states the reference lines it follows. What matters for parity
 * is the order of every fp32 operation that feeds an int8 quantization, the KV
 * cache or the logits; those orders are spelled out in the comments. Build with
 * -fno-fast-math -ffp-contract=off (oracle/Makefile; -O3, which vectorizes only
 * independent lanes and integer sums without -ffast-math) so the compiler neither
 * fuses multiply-adds nor reorders a floating-point sum. Rows of a matmul, heads
 * of attention and the tokens of a prefill chunk are independent, so splitting
 * them over threads does not change any result.
 *
 * Parity pin: see ember_oracle.h.
 */
#ifndef _DEFAULT_SOURCE
#define _DEFAULT_SOURCE
#endif
#include "ember_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <pthread.h>

enum { DT_F32 = 0, DT_Q8 = 1, DT_Q4 = 2 };
#define QB 32

#pragma pack(push, 1)
typedef struct {
    char magic[4]; uint32_t version; uint64_t header_bytes;
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab_size, max_seq_len;
    float rope_theta, norm_eps; uint32_t flags; int32_t rope_style;
    int32_t bos, eos, eos2, n_tensors, tok_type, top_k; float temp, top_p;
    uint64_t tok_off, tok_size, table_off, table_size; uint8_t reserved[128];
} Hdr;
typedef struct { char name[48]; int32_t dtype, ndim, shape[4]; uint64_t offset, nbytes; } Ten;
typedef struct { uint16_t d; int8_t qs[QB]; } Q8;
typedef struct { uint16_t d; uint8_t qs[QB / 2]; } Q4;
#pragma pack(pop)

static void fatal(const char *msg) { fprintf(stderr, "oracle: %s\n", msg); exit(1); }

/* ---- a small fork-join pool: splits [0,n) into equal slices ----------------- */
typedef void (*RangeFn)(void *ctx, int i0, int i1);
static int g_threads = 1;
static pthread_t g_workers[64];
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t g_go = PTHREAD_COND_INITIALIZER, g_done = PTHREAD_COND_INITIALIZER;
static unsigned long g_round = 0;
static int g_pending = 0, g_n = 0;
static RangeFn g_fn;
static void *g_ctx;

static void run_slice(int id) {
    long lo = (long)g_n * id / g_threads, hi = (long)g_n * (id + 1) / g_threads;
    if (hi > lo) g_fn(g_ctx, (int)lo, (int)hi);
}

static void *worker(void *arg) {
    int id = (int)(long)arg;
    unsigned long seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_mu);
        while (g_round == seen) pthread_cond_wait(&g_go, &g_mu);
        seen = g_round;
        pthread_mutex_unlock(&g_mu);
        run_slice(id);
        pthread_mutex_lock(&g_mu);
        if (--g_pending == 0) pthread_cond_signal(&g_done);
        pthread_mutex_unlock(&g_mu);
    }
    return NULL;
}

void orc_set_threads(int n) {
    if (g_threads > 1 || n <= 1) return;          /* set once per process */
    if (n > 64) n = 64;
    int made = 1;
    for (int i = 1; i < n; i++)
        if (pthread_create(&g_workers[i], NULL, worker, (void *)(long)i) == 0) made++;
        else break;
    g_threads = made;
}

static void par_for(RangeFn fn, void *ctx, int n, int parallel) {
    if (g_threads <= 1 || !parallel) { fn(ctx, 0, n); return; }
    pthread_mutex_lock(&g_mu);
    g_fn = fn; g_ctx = ctx; g_n = n; g_pending = g_threads - 1; g_round++;
    pthread_cond_broadcast(&g_go);
    pthread_mutex_unlock(&g_mu);
    run_slice(0);
    pthread_mutex_lock(&g_mu);
    while (g_pending > 0) pthread_cond_wait(&g_done, &g_mu);
    pthread_mutex_unlock(&g_mu);
}

/* ---- fp16 (ref src/kernels.c:25-68) ---------------------------------------- */
float orc_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u, b;
    if (e == 31u) b = s | 0x7F800000u | (m << 13);
    else if (e) b = s | ((e + 112u) << 23) | (m << 13);
    else if (!m) b = s;
    else { int k = 0; while (!(m & 0x400u)) { m <<= 1; k++; } b = s | ((uint32_t)(113 - k) << 23) | ((m & 1023u) << 13); }
    float f; memcpy(&f, &b, 4); return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t s = (x >> 16) & 0x8000u, e = (x >> 23) & 255u, m = x & 0x7FFFFFu;
    if (e >= 143u) return (uint16_t)(s | 0x7C00u);
    if (e >= 113u) {
        uint32_t h = ((e - 112u) << 10) | (m >> 13), r = m & 0x1FFFu;
        if (r > 0x1000u || (r == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(s | h);
    }
    if (e < 102u) return (uint16_t)s;
    uint32_t full = m | 0x800000u, sh = 126u - e, h = full >> sh, r = full & ((1u << sh) - 1u);
    uint32_t half = 1u << (sh - 1u);
    if (r > half || (r == half && (h & 1u))) h++;
    return (uint16_t)(s | h);
}

/* ---- quantizers (ref src/kernels.c:73-115) ---------------------------------- */
void orc_quantize_q8_0(const float *x, void *out_blocks, int n) {
    Q8 *out = out_blocks;
    for (int b = 0; b < n / QB; b++) {
        const float *v = x + b * QB;
        float amax = 0.0f;
        for (int i = 0; i < QB; i++) { float a = fabsf(v[i]); if (a > amax) amax = a; }
        float d = amax / 127.0f;                 /* fp32 division */
        float id = d > 0.0f ? 1.0f / d : 0.0f;   /* reciprocal of the UNROUNDED d */
        out[b].d = orc_f32_to_f16(d);
        for (int i = 0; i < QB; i++) {
            long q = lroundf(v[i] * id);         /* half away from zero */
            out[b].qs[i] = (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
        }
    }
}

void orc_quantize_q4_0(const float *x, void *out_blocks, int n) {
    Q4 *out = out_blocks;
    for (int b = 0; b < n / QB; b++) {
        const float *v = x + b * QB;
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < QB; i++) { float a = fabsf(v[i]); if (a > amax) { amax = a; vmax = v[i]; } }
        float d = vmax / -8.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
        out[b].d = orc_f32_to_f16(d);
        for (int i = 0; i < QB / 2; i++) {
            int lo = (int)(v[i] * id + 8.5f), hi = (int)(v[i + QB / 2] * id + 8.5f);
            lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
            hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
            out[b].qs[i] = (uint8_t)(lo | (hi << 4));
        }
    }
}

/* ---- dot products (ref src/kernels.c:120-183, portable/scalar paths) ------- */
static float dot_f32(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];   /* product rounded, then added, in order */
    return s;
}

/* sum over blocks, in block order, of ((float)acc * d_w) * d_x */
static float dot_q8(const Q8 *w, const Q8 *x, int nb) {
    float s = 0.0f;
    for (int b = 0; b < nb; b++) {
        int32_t acc = 0;
        for (int i = 0; i < QB; i++) acc += (int32_t)w[b].qs[i] * (int32_t)x[b].qs[i];
        s += (float)acc * orc_f16_to_f32(w[b].d) * orc_f16_to_f32(x[b].d);
    }
    return s;
}

static float dot_q4(const Q4 *w, const Q8 *x, int nb) {
    float s = 0.0f;
    for (int b = 0; b < nb; b++) {
        int32_t acc = 0;
        for (int i = 0; i < QB / 2; i++)
            acc += ((int32_t)(w[b].qs[i] & 15) - 8) * x[b].qs[i] +
                   ((int32_t)(w[b].qs[i] >> 4) - 8) * x[b].qs[i + QB / 2];
        s += (float)acc * orc_f16_to_f32(w[b].d) * orc_f16_to_f32(x[b].d);
    }
    return s;
}

typedef struct { float *out; const void *x, *w; int dtype, n_in; } MM;

static void mm_slice(void *c, int r0, int r1) {
    const MM *a = c;
    int nb = a->n_in / QB;
    for (int r = r0; r < r1; r++) {
        if (a->dtype == DT_F32) a->out[r] = dot_f32((const float *)a->w + (size_t)r * a->n_in, a->x, a->n_in);
        else if (a->dtype == DT_Q8) a->out[r] = dot_q8((const Q8 *)a->w + (size_t)r * nb, a->x, nb);
        else a->out[r] = dot_q4((const Q4 *)a->w + (size_t)r * nb, a->x, nb);
    }
}

static void rows_matmul(float *out, const void *xin, const void *w, int dtype, int n_in, int d_out) {
    MM a = { out, xin, w, dtype, n_in };
    par_for(mm_slice, &a, d_out, (long)d_out * n_in >= 1L << 20);
}

/* ref src/kernels.c:207-220: quantize the activation once, then one dot per row */
void orc_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out,
                void *xq) {
    const void *xin = x;
    if (dtype != DT_F32) { orc_quantize_q8_0(x, xq, n_in); xin = xq; }
    rows_matmul(out, xin, w, dtype, n_in, d_out);
}

/* ref src/kernels.c:250-264: per token the same arithmetic as orc_matmul
 * (batch_matmul below: every column quantized into xq, one dot per row and
 * column) */
static void batch_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out, int n, Q8 *xq);

void orc_matmul_batch(float *out, const float *x, const void *w, int dtype, int n_in,
                      int d_out, int B, void *xq) {
    batch_matmul(out, x, w, dtype, n_in, d_out, B, (Q8 *)xq);
}

/* ---- model pieces (ref src/model.c:50-100) --------------------------------- */
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];          /* in index order */
    float scale = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i]; /* (x*scale)*w */
}

float orc_expf(float x) { return expf(x); }

static void softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

static void rope(float *v, int n, int hd, int pos, float theta, int neox) {
    for (int h = 0; h < n; h += hd)
        for (int i = 0; i < hd / 2; i++) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / hd);
            float ang = pos * freq;
            float c = cosf(ang), s = sinf(ang);
            int a = neox ? h + i : h + 2 * i, b = neox ? h + i + hd / 2 : h + 2 * i + 1;
            float v0 = v[a], v1 = v[b];
            v[a] = v0 * c - v1 * s;
            v[b] = v0 * s + v1 * c;
        }
}

/* ---- loader ----------------------------------------------------------------- */
typedef struct { const void *p; int dt; } W;

struct OrcModel {
    size_t size; const uint8_t *base; const Hdr *h; const Ten *t;
};

OrcModel *orc_load(const char *path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 256) { close(fd); return NULL; }
    void *b = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (b == MAP_FAILED) return NULL;
    OrcModel *m = calloc(1, sizeof(*m));
    m->size = (size_t)st.st_size; m->base = b; m->h = b;
    if (memcmp(m->h->magic, "EMBR", 4) != 0 || m->h->table_off + m->h->table_size > m->size) {
        munmap(b, m->size); free(m); return NULL;
    }
    m->t = (const Ten *)(m->base + m->h->table_off);
    return m;
}

void orc_free(OrcModel *m) { if (m) { munmap((void *)m->base, m->size); free(m); } }

static W tensor(const OrcModel *m, const char *fmt, int l) {
    char name[48];
    if (l >= 0) snprintf(name, sizeof(name), fmt, l); else snprintf(name, sizeof(name), "%s", fmt);
    W w = { NULL, DT_F32 };
    for (int i = 0; i < m->h->n_tensors; i++)
        if (strncmp(m->t[i].name, name, 48) == 0) {
            if (m->t[i].offset + m->t[i].nbytes <= m->size) { w.p = m->base + m->t[i].offset; w.dt = m->t[i].dtype; }
            break;
        }
    return w;
}

/* ---- state + forward (ref src/model.c:18-35, :120-193, :221-278, :362-414) -- */
struct OrcState {
    const OrcModel *m;
    int dim, hidden, L, nh, nkv, hd, kvd, vocab, ctx, f16kv, qkn, neox;
    float theta, eps;
    W emb, head; const float *fnorm;
    W *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    const float **an, **fn, **qn, **kn, **bq, **bk, **bv;
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
    void *kc, *vc;
    void *xq;
};

OrcState *orc_state_new(OrcModel *m, int ctx_len, int kv_fp16) {
    const Hdr *h = m->h;
    OrcState *s = calloc(1, sizeof(*s));
    s->m = m; s->dim = h->dim; s->hidden = h->hidden_dim; s->L = h->n_layers;
    s->nh = h->n_heads; s->nkv = h->n_kv_heads; s->hd = h->head_dim; s->kvd = s->nkv * s->hd;
    s->vocab = h->vocab_size; s->theta = h->rope_theta; s->eps = h->norm_eps;
    s->neox = h->rope_style == 1; s->qkn = (h->flags & 2u) != 0; s->f16kv = kv_fp16 != 0;
    s->ctx = (ctx_len > 0 && ctx_len < h->max_seq_len) ? ctx_len : h->max_seq_len;
    int L = s->L;
    s->wq = calloc(L, sizeof(W)); s->wk = calloc(L, sizeof(W)); s->wv = calloc(L, sizeof(W));
    s->wo = calloc(L, sizeof(W)); s->w1 = calloc(L, sizeof(W)); s->w2 = calloc(L, sizeof(W));
    s->w3 = calloc(L, sizeof(W));
    s->an = calloc(L, sizeof(float *)); s->fn = calloc(L, sizeof(float *));
    s->qn = calloc(L, sizeof(float *)); s->kn = calloc(L, sizeof(float *));
    s->bq = calloc(L, sizeof(float *)); s->bk = calloc(L, sizeof(float *)); s->bv = calloc(L, sizeof(float *));
    for (int l = 0; l < L; l++) {
        s->wq[l] = tensor(m, "layers.%d.wq", l); s->wk[l] = tensor(m, "layers.%d.wk", l);
        s->wv[l] = tensor(m, "layers.%d.wv", l); s->wo[l] = tensor(m, "layers.%d.wo", l);
        s->w1[l] = tensor(m, "layers.%d.w1", l); s->w2[l] = tensor(m, "layers.%d.w2", l);
        s->w3[l] = tensor(m, "layers.%d.w3", l);
        s->an[l] = tensor(m, "layers.%d.attn_norm", l).p; s->fn[l] = tensor(m, "layers.%d.ffn_norm", l).p;
        s->qn[l] = tensor(m, "layers.%d.q_norm", l).p; s->kn[l] = tensor(m, "layers.%d.k_norm", l).p;
        s->bq[l] = tensor(m, "layers.%d.wq_bias", l).p; s->bk[l] = tensor(m, "layers.%d.wk_bias", l).p;
        s->bv[l] = tensor(m, "layers.%d.wv_bias", l).p;
        if (!s->wq[l].p || !s->wk[l].p || !s->wv[l].p || !s->wo[l].p || !s->w1[l].p ||
            !s->w2[l].p || !s->w3[l].p || !s->an[l] || !s->fn[l]) fatal("missing layer tensor");
    }
    s->emb = tensor(m, "tok_embeddings", -1);
    s->fnorm = tensor(m, "final_norm", -1).p;
    s->head = (h->flags & 1u) ? s->emb : tensor(m, "lm_head", -1);
    if (!s->emb.p || !s->fnorm || !s->head.p) fatal("missing global tensor");
    int qd = s->nh * s->hd, wide = s->dim;
    if (s->hidden > wide) wide = s->hidden;
    if (qd > wide) wide = qd;
    s->x = calloc(s->dim, 4); s->xb = calloc(qd > s->dim ? qd : s->dim, 4); s->xb2 = calloc(s->dim, 4);
    s->hb = calloc(s->hidden, 4); s->hb2 = calloc(s->hidden, 4); s->q = calloc(qd, 4);
    s->k = calloc(s->kvd, 4); s->v = calloc(s->kvd, 4);
    s->att = calloc((size_t)s->nh * s->ctx, 4); s->logits = calloc(s->vocab, 4);
    size_t kvn = (size_t)L * s->ctx * s->kvd, es = s->f16kv ? 2 : 4;
    s->kc = calloc(kvn, es); s->vc = calloc(kvn, es);
    s->xq = calloc(wide / QB + 1, sizeof(Q8));
    if (!s->kc || !s->vc) fatal("out of memory for the KV cache");
    return s;
}

void orc_state_free(OrcState *s) {
    if (!s) return;
    free(s->wq); free(s->wk); free(s->wv); free(s->wo); free(s->w1); free(s->w2); free(s->w3);
    free(s->an); free(s->fn); free(s->qn); free(s->kn); free(s->bq); free(s->bk); free(s->bv);
    free(s->x); free(s->xb); free(s->xb2); free(s->hb); free(s->hb2); free(s->q); free(s->k);
    free(s->v); free(s->att); free(s->logits); free(s->kc); free(s->vc); free(s->xq); free(s);
}

int orc_state_ctx(const OrcState *s) { return s->ctx; }


/* fp16 -> fp32 of every half value, filled once (the widening is exact) */
static float g_f16[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void f16_table_init(void) {
    for (uint32_t i = 0; i < 65536u; i++) g_f16[i] = orc_f16_to_f32((uint16_t)i);
}

/* row of hd cached values at element offset `base`, widened to fp32 */
static const float *kv_row(const OrcState *s, const void *cache, size_t base, int hd, float *buf) {
    if (!s->f16kv) return (const float *)cache + base;
    const uint16_t *h = (const uint16_t *)cache + base;
    for (int i = 0; i < hd; i++) buf[i] = g_f16[h[i]];
    return buf;
}

/* One query position over the cache for one head (ref src/model.c:221-259):
 * scores sc_t = sum_i q_i*k_t,i in index order, then * inv_sqrt; softmax; then
 * out_i = sum_t w_t*v_t,i in position order. The score chains of different
 * positions are independent, so eight of them advance side by side here (keys
 * staged dimension-major); each one still adds its products in index order.
 * `att` is scratch of pos+1 floats; hd <= 256. */
static void attend_one(const OrcState *s, int l, int pos, const float *qh, int h, float *att, float *out) {
    int hd = s->hd, kvd = s->kvd, mul = s->nh / s->nkv, kvh = h / mul;
    size_t lo = (size_t)l * s->ctx * kvd;
    float inv_sqrt = 1.0f / sqrtf((float)hd);
    float tile[256][8], buf[256];
    pthread_once(&g_f16_once, f16_table_init);
    int t = 0;
    for (; t + 8 <= pos + 1; t += 8) {
        for (int j = 0; j < 8; j++) {
            const float *kr = kv_row(s, s->kc, lo + (size_t)(t + j) * kvd + (size_t)kvh * hd, hd, buf);
            for (int i = 0; i < hd; i++) tile[i][j] = kr[i];
        }
        float sc[8] = { 0, 0, 0, 0, 0, 0, 0, 0 };
        for (int i = 0; i < hd; i++)
            for (int j = 0; j < 8; j++) sc[j] += qh[i] * tile[i][j];
        for (int j = 0; j < 8; j++) att[t + j] = sc[j] * inv_sqrt;
    }
    for (; t <= pos; t++) {
        const float *kr = kv_row(s, s->kc, lo + (size_t)t * kvd + (size_t)kvh * hd, hd, buf);
        float sc = 0.0f;
        for (int i = 0; i < hd; i++) sc += qh[i] * kr[i];
        att[t] = sc * inv_sqrt;
    }
    softmax(att, pos + 1);
    for (int i = 0; i < hd; i++) out[i] = 0.0f;
    for (t = 0; t <= pos; t++) {
        float w = att[t];
        const float *vr = kv_row(s, s->vc, lo + (size_t)t * kvd + (size_t)kvh * hd, hd, buf);
        for (int i = 0; i < hd; i++) out[i] += w * vr[i];
    }
}

typedef struct { OrcState *s; int l, pos; } AT;

static void attend_heads(void *c, int h0, int h1) {
    const AT *a = c;
    OrcState *s = a->s;
    for (int h = h0; h < h1; h++)
        attend_one(s, a->l, a->pos, s->q + h * s->hd, h, s->att + (size_t)h * s->ctx, s->xb + h * s->hd);
}

static void attend(OrcState *s, int l, int pos) {
    AT a = { s, l, pos };
    par_for(attend_heads, &a, s->nh, (long)s->nh * (pos + 1) * s->hd >= 1L << 17);
}

static void embed(const OrcState *s, int tok, float *out) {
    if (s->emb.dt == DT_F32) { memcpy(out, (const float *)s->emb.p + (size_t)tok * s->dim, 4 * (size_t)s->dim); return; }
    const Q8 *row = (const Q8 *)s->emb.p + (size_t)tok * (s->dim / QB);
    for (int b = 0; b < s->dim / QB; b++) {
        float d = orc_f16_to_f32(row[b].d);
        for (int i = 0; i < QB; i++) out[b * QB + i] = row[b].qs[i] * d;
    }
}

float *orc_forward(OrcState *s, int tok, int pos) {
    int dim = s->dim, hd = s->hd, nh = s->nh, kvd = s->kvd, qd = nh * hd;
    if (tok < 0 || tok >= s->vocab || pos < 0 || pos >= s->ctx) fatal("token or position out of range");
    embed(s, tok, s->x);
    for (int l = 0; l < s->L; l++) {
        orc_rmsnorm(s->xb, s->x, s->an[l], dim, s->eps);
        orc_matmul(s->q, s->xb, s->wq[l].p, s->wq[l].dt, dim, qd, s->xq);
        orc_matmul(s->k, s->xb, s->wk[l].p, s->wk[l].dt, dim, kvd, s->xq);
        orc_matmul(s->v, s->xb, s->wv[l].p, s->wv[l].dt, dim, kvd, s->xq);
        if (s->bq[l]) for (int i = 0; i < qd; i++) s->q[i] += s->bq[l][i];
        if (s->bk[l]) for (int i = 0; i < kvd; i++) s->k[i] += s->bk[l][i];
        if (s->bv[l]) for (int i = 0; i < kvd; i++) s->v[i] += s->bv[l][i];
        if (s->qkn && s->qn[l]) {
            for (int h = 0; h < nh; h++) orc_rmsnorm(s->q + h * hd, s->q + h * hd, s->qn[l], hd, s->eps);
            for (int h = 0; h < s->nkv; h++) orc_rmsnorm(s->k + h * hd, s->k + h * hd, s->kn[l], hd, s->eps);
        }
        rope(s->q, qd, hd, pos, s->theta, s->neox);
        rope(s->k, kvd, hd, pos, s->theta, s->neox);
        size_t off = ((size_t)l * s->ctx + pos) * kvd;
        for (int i = 0; i < kvd; i++) {          /* kv_store, ref src/model.c:39-48 */
            if (s->f16kv) {
                ((uint16_t *)s->kc)[off + i] = orc_f32_to_f16(s->k[i]);
                ((uint16_t *)s->vc)[off + i] = orc_f32_to_f16(s->v[i]);
            } else {
                ((float *)s->kc)[off + i] = s->k[i];
                ((float *)s->vc)[off + i] = s->v[i];
            }
        }
        attend(s, l, pos);
        orc_matmul(s->xb2, s->xb, s->wo[l].p, s->wo[l].dt, qd, dim, s->xq);
        for (int i = 0; i < dim; i++) s->x[i] += s->xb2[i];
        orc_rmsnorm(s->xb, s->x, s->fn[l], dim, s->eps);
        orc_matmul(s->hb, s->xb, s->w1[l].p, s->w1[l].dt, dim, s->hidden, s->xq);
        orc_matmul(s->hb2, s->xb, s->w3[l].p, s->w3[l].dt, dim, s->hidden, s->xq);
        for (int i = 0; i < s->hidden; i++) {   /* SiLU(g) * u, ref src/model.c:403-406 */
            float g = s->hb[i];
            s->hb[i] = g / (1.0f + expf(-g)) * s->hb2[i];
        }
        orc_matmul(s->xb, s->hb, s->w2[l].p, s->w2[l].dt, s->hidden, dim, s->xq);
        for (int i = 0; i < dim; i++) s->x[i] += s->xb[i];
    }
    orc_rmsnorm(s->x, s->x, s->fnorm, dim, s->eps);
    orc_matmul(s->logits, s->x, s->head.p, s->head.dt, dim, s->vocab, s->xq);
    return s->logits;
}

/* ---- batched prefill (ref src/model.c:283-360) ------------------------------
 * The reference's prefill runs every layer over all n tokens at once: each
 * matmul quantizes every token's activation and streams each weight row once for
 * all tokens (ember_matmul_batch, ref src/kernels.c:227-264, the same per-(row,
 * token) dot as ember_matmul); norms, bias, QK-norm, RoPE and the KV store run
 * per token; then attention per token, token b reading positions <= start+b;
 * only the last token's logits are computed. Every token's arithmetic is the one
 * orc_forward performs. Tokens go through in chunks of PF_CHUNK, which changes
 * nothing: a chunk's attention reads only positions written before it or by its
 * own KV store. */
enum { PF_CHUNK = 256 };

typedef struct { float *out; const Q8 *xq; const void *w; int dtype, n_in, d_out, n; const float *xf; } BMM;

/* int8 dot of one block pair: exact in any order */
static int32_t block_dot_q8(const int8_t *w, const int8_t *x) {
    int32_t acc = 0;
    for (int i = 0; i < QB; i++) acc += (int32_t)w[i] * (int32_t)x[i];
    return acc;
}

static int32_t block_dot_q4(const uint8_t *w, const int8_t *x) {
    int32_t acc = 0;
    for (int i = 0; i < QB / 2; i++)
        acc += ((int32_t)(w[i] & 15) - 8) * x[i] + ((int32_t)(w[i] >> 4) - 8) * x[i + QB / 2];
    return acc;
}

/* Per (row, token): the chain of dot_q8 / dot_q4, sum over blocks in block order
 * of ((float)acc * d_w) * d_x, with the fp16 scales widened once per row and per
 * token (the widening is exact, so this changes no result). */
static void bmm_slice(void *c, int r0, int r1) {
    const BMM *a = c;
    int nb = a->n_in / QB;
    float *dw = malloc(sizeof(float) * (size_t)(nb + 1));
    float *dx = malloc(sizeof(float) * (size_t)a->n * (nb + 1));
    if (!dw || !dx) fatal("out of memory");
    if (a->dtype != DT_F32)
        for (int b = 0; b < a->n; b++)
            for (int k = 0; k < nb; k++) dx[(size_t)b * nb + k] = orc_f16_to_f32(a->xq[(size_t)b * nb + k].d);
    for (int r = r0; r < r1; r++) {
        if (a->dtype == DT_F32) {
            for (int b = 0; b < a->n; b++)
                a->out[(size_t)b * a->d_out + r] =
                    dot_f32((const float *)a->w + (size_t)r * a->n_in, a->xf + (size_t)b * a->n_in, a->n_in);
            continue;
        }
        const Q8 *w8 = (const Q8 *)a->w + (size_t)r * nb;
        const Q4 *w4 = (const Q4 *)a->w + (size_t)r * nb;
        for (int k = 0; k < nb; k++) dw[k] = orc_f16_to_f32(a->dtype == DT_Q8 ? w8[k].d : w4[k].d);
        for (int b = 0; b < a->n; b++) {
            const Q8 *xb = a->xq + (size_t)b * nb;
            const float *dxb = dx + (size_t)b * nb;
            float s = 0.0f;
            for (int k = 0; k < nb; k++) {
                int32_t acc = a->dtype == DT_Q8 ? block_dot_q8(w8[k].qs, xb[k].qs) : block_dot_q4(w4[k].qs, xb[k].qs);
                s += (float)acc * dw[k] * dxb[k];
            }
            a->out[(size_t)b * a->d_out + r] = s;
        }
    }
    free(dw);
    free(dx);
}

/* out[b][d_out] = W x[b] for b < n; xq: n * (n_in/32) Q8 blocks of scratch */
static void batch_matmul(float *out, const float *x, const void *w, int dtype, int n_in, int d_out, int n, Q8 *xq) {
    int nb = n_in / QB;
    if (dtype != DT_F32)
        for (int b = 0; b < n; b++) orc_quantize_q8_0(x + (size_t)b * n_in, xq + (size_t)b * nb, n_in);
    BMM a = { out, xq, w, dtype, n_in, d_out, n, x };
    par_for(bmm_slice, &a, d_out, 1);
}

/* Attention of a chunk of n query tokens (positions start..start+n-1), one head
 * per work item: the same per-(token, head) arithmetic as attend_one -- every
 * score chain over the dimensions in index order, softmax, every output chain
 * over the positions in order -- with the loops arranged so that each staged key
 * tile and each value row serves all tokens that attend to it. */
typedef struct { OrcState *s; int l, start, n; const float *Q; float *O; } BAT;

static void battend_head(void *c, int h0, int h1) {
    const BAT *a = c;
    OrcState *s = a->s;
    int hd = s->hd, kvd = s->kvd, mul = s->nh / s->nkv, qd = s->nh * hd, n = a->n, start = a->start;
    int T = start + n;                       /* positions the last token attends: 0..T-1 */
    size_t lo = (size_t)a->l * s->ctx * kvd;
    float inv_sqrt = 1.0f / sqrtf((float)hd);
    float *att = malloc(sizeof(float) * (size_t)n * T);
    if (!att) fatal("out of memory");
    float tile[256][8], buf[256];
    pthread_once(&g_f16_once, f16_table_init);
    for (int h = h0; h < h1; h++) {
        int kvh = h / mul;
        /* scores: token b attends positions 0..start+b */
        int t = 0;
        for (; t + 8 <= T; t += 8) {
            for (int j = 0; j < 8; j++) {
                const float *kr = kv_row(s, s->kc, lo + (size_t)(t + j) * kvd + (size_t)kvh * hd, hd, buf);
                for (int i = 0; i < hd; i++) tile[i][j] = kr[i];
            }
            int b0 = t + 7 - start;          /* first token that sees all 8 positions */
            if (b0 < 0) b0 = 0;
            for (int b = b0; b < n; b++) {
                const float *qh = a->Q + (size_t)b * qd + h * hd;
                float sc[8] = { 0, 0, 0, 0, 0, 0, 0, 0 };
                for (int i = 0; i < hd; i++)
                    for (int j = 0; j < 8; j++) sc[j] += qh[i] * tile[i][j];
                for (int j = 0; j < 8; j++) att[(size_t)b * T + t + j] = sc[j] * inv_sqrt;
            }
            for (int b = 0; b < b0 && b < n; b++)      /* tokens that see only part of the tile */
                for (int j = 0; j < 8 && t + j <= start + b; j++) {
                    const float *qh = a->Q + (size_t)b * qd + h * hd;
                    float sc = 0.0f;
                    for (int i = 0; i < hd; i++) sc += qh[i] * tile[i][j];
                    att[(size_t)b * T + t + j] = sc * inv_sqrt;
                }
        }
        for (; t < T; t++) {
            const float *kr = kv_row(s, s->kc, lo + (size_t)t * kvd + (size_t)kvh * hd, hd, buf);
            for (int b = t - start < 0 ? 0 : t - start; b < n; b++) {
                const float *qh = a->Q + (size_t)b * qd + h * hd;
                float sc = 0.0f;
                for (int i = 0; i < hd; i++) sc += qh[i] * kr[i];
                att[(size_t)b * T + t] = sc * inv_sqrt;
            }
        }
        for (int b = 0; b < n; b++) {
            softmax(att + (size_t)b * T, start + b + 1);
            float *out = a->O + (size_t)b * qd + h * hd;
            for (int i = 0; i < hd; i++) out[i] = 0.0f;
        }
        /* outputs: out_b,i += w_b,t * v_t,i for t in order */
        for (t = 0; t < T; t++) {
            const float *vr = kv_row(s, s->vc, lo + (size_t)t * kvd + (size_t)kvh * hd, hd, buf);
            for (int b = t - start < 0 ? 0 : t - start; b < n; b++) {
                float w = att[(size_t)b * T + t];
                float *out = a->O + (size_t)b * qd + h * hd;
                for (int i = 0; i < hd; i++) out[i] += w * vr[i];
            }
        }
    }
    free(att);
}

static void prefill_chunk(OrcState *s, const int *ids, int n, int start, float *X, float *Xn, float *Tmp,
                          float *Q, float *K, float *V, float *O, float *H1, float *H2, Q8 *xq) {
    int dim = s->dim, hd = s->hd, nh = s->nh, kvd = s->kvd, qd = nh * hd, hid = s->hidden;
    for (int b = 0; b < n; b++) embed(s, ids[b], X + (size_t)b * dim);
    for (int l = 0; l < s->L; l++) {
        for (int b = 0; b < n; b++) orc_rmsnorm(Xn + (size_t)b * dim, X + (size_t)b * dim, s->an[l], dim, s->eps);
        batch_matmul(Q, Xn, s->wq[l].p, s->wq[l].dt, dim, qd, n, xq);
        batch_matmul(K, Xn, s->wk[l].p, s->wk[l].dt, dim, kvd, n, xq);
        batch_matmul(V, Xn, s->wv[l].p, s->wv[l].dt, dim, kvd, n, xq);
        for (int b = 0; b < n; b++) {
            float *qb = Q + (size_t)b * qd, *kb = K + (size_t)b * kvd, *vb = V + (size_t)b * kvd;
            int pos = start + b;
            if (s->bq[l]) for (int i = 0; i < qd; i++) qb[i] += s->bq[l][i];
            if (s->bk[l]) for (int i = 0; i < kvd; i++) kb[i] += s->bk[l][i];
            if (s->bv[l]) for (int i = 0; i < kvd; i++) vb[i] += s->bv[l][i];
            if (s->qkn && s->qn[l]) {
                for (int h = 0; h < nh; h++) orc_rmsnorm(qb + h * hd, qb + h * hd, s->qn[l], hd, s->eps);
                for (int h = 0; h < s->nkv; h++) orc_rmsnorm(kb + h * hd, kb + h * hd, s->kn[l], hd, s->eps);
            }
            rope(qb, qd, hd, pos, s->theta, s->neox);
            rope(kb, kvd, hd, pos, s->theta, s->neox);
            size_t off = ((size_t)l * s->ctx + pos) * kvd;
            for (int i = 0; i < kvd; i++) {
                if (s->f16kv) {
                    ((uint16_t *)s->kc)[off + i] = orc_f32_to_f16(kb[i]);
                    ((uint16_t *)s->vc)[off + i] = orc_f32_to_f16(vb[i]);
                } else {
                    ((float *)s->kc)[off + i] = kb[i];
                    ((float *)s->vc)[off + i] = vb[i];
                }
            }
        }
        BAT at = { s, l, start, n, Q, O };
        par_for(battend_head, &at, nh, 1);
        batch_matmul(Tmp, O, s->wo[l].p, s->wo[l].dt, qd, dim, n, xq);
        for (size_t i = 0; i < (size_t)n * dim; i++) X[i] += Tmp[i];
        for (int b = 0; b < n; b++) orc_rmsnorm(Xn + (size_t)b * dim, X + (size_t)b * dim, s->fn[l], dim, s->eps);
        batch_matmul(H1, Xn, s->w1[l].p, s->w1[l].dt, dim, hid, n, xq);
        batch_matmul(H2, Xn, s->w3[l].p, s->w3[l].dt, dim, hid, n, xq);
        for (size_t i = 0; i < (size_t)n * hid; i++) {
            float g = H1[i];
            H1[i] = g / (1.0f + expf(-g)) * H2[i];
        }
        batch_matmul(Tmp, H1, s->w2[l].p, s->w2[l].dt, hid, dim, n, xq);
        for (size_t i = 0; i < (size_t)n * dim; i++) X[i] += Tmp[i];
    }
}

float *orc_prefill(OrcState *s, const int *ids, int n, int start) {
    if (n <= 0) return s->logits;
    if (start < 0 || start + n > s->ctx) fatal("prefill past the context");
    for (int b = 0; b < n; b++)
        if (ids[b] < 0 || ids[b] >= s->vocab) fatal("token id out of range");
    int c = n < PF_CHUNK ? n : PF_CHUNK;
    int dim = s->dim, qd = s->nh * s->hd, wide = dim;
    if (s->hidden > wide) wide = s->hidden;
    if (qd > wide) wide = qd;
    float *X = malloc(sizeof(float) * (size_t)c * dim), *Xn = malloc(sizeof(float) * (size_t)c * dim);
    float *Tmp = malloc(sizeof(float) * (size_t)c * dim), *Q = malloc(sizeof(float) * (size_t)c * qd);
    float *K = malloc(sizeof(float) * (size_t)c * s->kvd), *V = malloc(sizeof(float) * (size_t)c * s->kvd);
    float *O = malloc(sizeof(float) * (size_t)c * qd), *H1 = malloc(sizeof(float) * (size_t)c * s->hidden);
    float *H2 = malloc(sizeof(float) * (size_t)c * s->hidden);
    Q8 *xq = malloc(sizeof(Q8) * (size_t)c * (wide / QB + 1));
    if (!X || !Xn || !Tmp || !Q || !K || !V || !O || !H1 || !H2 || !xq) fatal("out of memory");
    int last = 0;
    for (int b0 = 0; b0 < n; b0 += c) {
        int m = n - b0 < c ? n - b0 : c;
        prefill_chunk(s, ids + b0, m, start + b0, X, Xn, Tmp, Q, K, V, O, H1, H2, xq);
        last = m - 1;
    }
    orc_rmsnorm(s->x, X + (size_t)last * dim, s->fnorm, dim, s->eps);
    orc_matmul(s->logits, s->x, s->head.p, s->head.dt, dim, s->vocab, s->xq);
    free(X); free(Xn); free(Tmp); free(Q); free(K); free(V); free(O); free(H1); free(H2); free(xq);
    return s->logits;
}

/* first index of the strict maximum (ref src/sample.c:114-118) */
int orc_argmax(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}

/* ---- the sampler (ref src/sample.c:76-175), over host logits, in place ----
 * Penalties over hist[0..hist_len) in array order; temperature <= 0: the first
 * index of the maximum; else logits / temperature, softmax (glibc expf, the
 * sum in index order, divide), candidates sorted by descending probability with
 * the C library's qsort and the reference's comparator, top_k, min_p, top_p,
 * then r = rng_f32 * cutoff and the first candidate whose running sum exceeds r.
 * *rng is the xorshift64* state (advanced once when temperature > 0). */
typedef struct { float prob; int idx; } OrcCand;

static int orc_cmp_desc(const void *a, const void *b) {
    float pa = ((const OrcCand *)a)->prob, pb = ((const OrcCand *)b)->prob;
    return (pa < pb) - (pa > pb);
}

int orc_sample(float *logits, int n, float temperature, float top_p, int top_k, float min_p,
               float repeat_penalty, float presence_penalty, float frequency_penalty, uint64_t *rng,
               const int *hist, int hist_len) {
    int has_rep = repeat_penalty != 1.0f, has_freq = frequency_penalty != 0.0f, has_pres = presence_penalty != 0.0f;
    if (hist && hist_len > 0 && (has_rep || has_freq || has_pres)) {
        for (int i = 0; i < hist_len; i++) {
            int t = hist[i];
            if (t < 0 || t >= n) continue;
            int first = 1;
            for (int j = 0; j < i; j++) if (hist[j] == t) { first = 0; break; }
            if (first) {
                if (has_rep) logits[t] = logits[t] > 0.0f ? logits[t] / repeat_penalty : logits[t] * repeat_penalty;
                if (has_pres) logits[t] -= presence_penalty;
            }
            if (has_freq) logits[t] -= frequency_penalty;
        }
    }
    if (temperature <= 0.0f) return orc_argmax(logits, n);
    for (int i = 0; i < n; i++) logits[i] /= temperature;
    float max = logits[orc_argmax(logits, n)];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { logits[i] = expf(logits[i] - max); sum += logits[i]; }
    for (int i = 0; i < n; i++) logits[i] /= sum;
    OrcCand *cand = malloc(sizeof(OrcCand) * (size_t)n);
    if (!cand) fatal("out of memory");
    for (int i = 0; i < n; i++) { cand[i].prob = logits[i]; cand[i].idx = i; }
    qsort(cand, (size_t)n, sizeof(OrcCand), orc_cmp_desc);
    int m = n;
    if (top_k > 0 && top_k < m) m = top_k;
    if (min_p > 0.0f && min_p < 1.0f) {
        float thresh = min_p * cand[0].prob;
        int keep = 1;
        while (keep < m && cand[keep].prob >= thresh) keep++;
        m = keep;
    }
    float cutoff;
    if (top_p > 0.0f && top_p < 1.0f) {
        float cum = 0.0f;
        int last = m - 1;
        for (int i = 0; i < m; i++) { cum += cand[i].prob; if (cum >= top_p) { last = i; break; } }
        m = last + 1;
        cutoff = cum;
    } else {
        cutoff = 0.0f;
        for (int i = 0; i < m; i++) cutoff += cand[i].prob;
    }
    uint64_t x = *rng;
    x ^= x >> 12; x ^= x << 25; x ^= x >> 27;
    *rng = x;
    float u = (float)((uint32_t)((x * 0x2545F4914F6CDD1DULL) >> 32) >> 8) / 16777216.0f;
    float r = u * cutoff, cum = 0.0f;
    int chosen = cand[m - 1].idx;
    for (int i = 0; i < m; i++) { cum += cand[i].prob; if (r < cum) { chosen = cand[i].idx; break; } }
    free(cand);
    return chosen;
}
