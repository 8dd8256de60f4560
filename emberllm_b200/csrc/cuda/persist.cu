// persist.cu — host side of the persistent token step (persist.cuh): whether a
// state can use it, its shared-memory plan, its hand-off buffers, and the
// cooperative launch that runs one forward step or a whole greedy run.
#include <cuda_runtime.h>

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "persist.cuh"
#include "runtime_internal.cuh"

using namespace emb;

namespace emb {

struct PState {
    PArgs a;                  // everything but n_steps / out_tokens
    size_t smem = 0;
    int grid = 0;
    uint32_t tag = 1;         // host copy of the next tag base (ctl[CTL_TAG])
    uint32_t tag_stride = 0;
    size_t words_bytes = 0;
    unsigned long long *words = nullptr;
};

}  // namespace emb

static int env_int(const char *name, int dflt) {
    const char *e = getenv(name);
    return e && *e ? atoi(e) : dflt;
}

static size_t al16(size_t n) { return (n + 15) / 16 * 16; }

// rows of one piece: quant rows plus a 16-byte-rounded scale window per matrix
static int rows_per_piece(int dtype, int cols, int nmat, int cap) {
    const int qrb = dtype == EMBER_DT_Q4_0 ? cols / 2 : cols, sb = cols / 32 * 2;
    int n = cap;
    while (n > 1 && (size_t)nmat * ((size_t)n * qrb + (size_t)n * sb + 30) > (size_t)P_SLOT) n--;
    return n;
}

// Why a state cannot take the persistent path, or NULL when it can.
static const char *persist_blocker(const EmberCudaState *s) {
    const EmberCudaModel *m = s->m;
    // opt-in: measured slower than the graph step on B200 (its per-stage
    // latencies exceed the launch overheads it saves)
    if (env_int("EMBER_PERSIST", 0) == 0) return "not requested (EMBER_PERSIST=1 selects it)";
    const int dt = m->layers.empty() ? -1 : m->layers[0].wq.dtype;
    if (dt != EMBER_DT_Q8_0 && dt != EMBER_DT_Q4_0) return "layer weights are not Q8_0/Q4_0";
    for (const DevLayer &L : m->layers) {
        const DevMat *ms[7] = {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3};
        for (const DevMat *d : ms)
            if (d->dtype != dt) return "mixed layer weight types";
    }
    if (m->tok_emb.dtype != EMBER_DT_Q8_0) return "the embedding is not Q8_0";
    if (m->lm_head.dtype != EMBER_DT_Q8_0 && m->lm_head.dtype != EMBER_DT_Q4_0) return "lm_head is not quantized";
    const int hd = m->head_dim, qd = m->n_heads * hd, G = m->n_sm - m->n_heads;
    if (m->dim % 32 || m->hidden % 32 || hd % 32 || 3 * hd > PT || m->n_heads % m->n_kv) return "shapes";
    if (m->dim > 4 * PT || qd / 4 + qd / 32 > 4 * PT || m->hidden / 4 + m->hidden / 32 > 4 * PT) return "too wide";
    if (m->n_heads > m->n_sm / 2) return "too many heads for the SMs";
    if (m->n_layers > P_MAXL) return "too many layers";
    // Every GEMV CTA must own at least one q/k/v row: each one's S1 outputs of
    // layer l+1 then depend on its having read every hand-off word of layer l,
    // so no word is rewritten before all its readers are done with it.
    if (qd + 2 * m->n_kv * hd < G) return "fewer q/k/v rows than GEMV CTAs";
    if ((qd + 2 * m->n_kv * hd + G - 1) / G > 64) return "too many q/k/v rows per CTA";
    return nullptr;
}

// why the last state creation did not take the persistent step ("" when it did)
static char g_persist_why[128] = "";

static int persist_no(const char *why) {
    snprintf(g_persist_why, sizeof(g_persist_why), "%s", why);
    if (env_int("EMBER_PERSIST_VERBOSE", 0)) fprintf(stderr, "ember: persistent step not used: %s\n", why);
    return 0;
}

extern "C" int ember_cuda_state_persistent(const EmberCudaState *s, const char **why) {
    if (why) *why = s->ps ? "" : g_persist_why;
    return s->ps != nullptr;
}

int emb::persist_init(EmberCudaState *s) {
    EmberCudaModel *m = s->m;
    if (const char *why = persist_blocker(s)) return persist_no(why);
    const int hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
    const int G = m->n_sm - m->n_heads;
    const int es = s->kv_fp16 ? 2 : 4;
    PArgs a;
    memset(&a, 0, sizeof(a));
    a.wdtype = m->layers[0].wq.dtype;
    a.dim = m->dim; a.hidden = m->hidden; a.L = m->n_layers; a.nh = m->n_heads; a.nkv = m->n_kv; a.hd = hd;
    a.vocab = m->vocab; a.ctx = s->ctx; a.kstride = s->kstride; a.neox = m->rope_neox; a.qk_norm = m->qk_norm;
    a.kv16 = s->kv_fp16; a.eps = m->eps; a.n_att = m->n_heads;
    a.emb_q = m->tok_emb.q; a.emb_s = m->tok_emb.s;
    a.head_q = m->lm_head.q; a.head_s = m->lm_head.s; a.head_dtype = m->lm_head.dtype;
    a.final_norm = m->final_norm;
    a.kc = s->kc; a.vc = s->vc; a.k_layer_elems = s->k_layer_elems; a.v_layer_elems = s->v_layer_elems;
    a.rope = s->rope; a.logits = s->logits; a.ctl = s->ctl;
    a.ex = m->ex;
    a.spin_limit = (uint32_t)env_int("EMBER_WAIT_POLLS", 1 << 22);
    a.poll_ns = (uint32_t)env_int("EMBER_POLL_NS", 200);
    // pieces
    a.rp_qkv = rows_per_piece(a.wdtype, m->dim, 1, 32);
    a.rp_wo = rows_per_piece(a.wdtype, qd, 1, 32);
    a.rp_w2 = rows_per_piece(a.wdtype, m->hidden, 1, 32);
    a.rp_head = rows_per_piece(m->lm_head.dtype, m->dim, 1, 32);
    a.pp_w13 = 32;
    while (a.pp_w13 > 1 && rows_per_piece(a.wdtype, m->dim, 2, a.pp_w13) < a.pp_w13) a.pp_w13 /= 2;
    {
        auto cdiv = [](long x, long y) { return (int)((x + y - 1) / y); };
        const int per_qkv = cdiv(qd + 2 * kvd, G), per_x = cdiv(m->dim, G), per_b = cdiv(m->hidden / 32, G);
        const int per_v = cdiv(m->vocab, G);
        const int pieces = cdiv(per_qkv, a.rp_qkv) + 3 + cdiv(per_x, a.rp_wo) + 1 + per_b * (32 / a.pp_w13) +
                           cdiv(per_x, a.rp_w2) + 1 + cdiv(per_v, a.rp_head) + 1;
        if (pieces > 2 * P_MAXPIECES) return persist_no("too many weight pieces per CTA");
    }
    // GEMV shared memory
    const int nbmax = (m->hidden > qd ? (m->hidden > m->dim ? m->hidden : m->dim) : (qd > m->dim ? qd : m->dim)) / 32;
    size_t off = (size_t)P_NSLOT * P_SLOT;
    a.g_xf = off; off += al16((size_t)m->dim * 4);
    a.g_sq = off; off += al16((size_t)m->dim * 4);
    a.g_xq = off; off += al16((size_t)nbmax * 32);
    a.g_xd = off; off += al16((size_t)nbmax * 4);
    size_t pfl = 2 * (size_t)G;
    auto pmax = [&](size_t rows, int cols) { size_t v = rows * (size_t)((cols / 32) | 1); if (v > pfl) pfl = v; };
    pmax(a.rp_qkv, m->dim); pmax(a.rp_wo, qd); pmax(2 * (size_t)a.pp_w13, m->dim); pmax(a.rp_w2, m->hidden);
    pmax(a.rp_head, m->dim);
    a.g_p = off; off += al16(pfl * 4);
    a.g_rowsum = off; off += 64 * 4;
    a.g_h = off; off += 32 * 4;
    a.g_xown = off; off += al16((size_t)((m->dim + G - 1) / G) * 4);
    a.g_nw = off; off += al16((size_t)m->dim * 16);      // two layers' attn + ffn norms
    a.g_bias = off; off += 2 * 64 * 4;                    // two layers' q/k/v biases of this CTA
    const size_t g_bytes = off;
    // the dynamic shared memory every CTA gets: the device's opt-in maximum
    // minus the kernel's static shared memory
    int optin = 0;
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    cudaFuncAttributes fa;
    if (s->kv_fp16) CK(cudaFuncGetAttributes(&fa, ember_persist_kernel<__half>));
    else CK(cudaFuncGetAttributes(&fa, ember_persist_kernel<float>));
    const size_t dyn = ((size_t)optin - fa.sharedSizeBytes - 256) / 128 * 128;
    if (g_bytes > dyn) return persist_no("the GEMV shared-memory plan does not fit");
    // attention: keys of the whole context, then values, then the scores
    a.kcap = (s->ctx + 7) / 8 * 8;
    a.k_bytes = (size_t)hd * a.kcap * es;
    a.v_off = al16(a.k_bytes);
    const size_t att_bytes = al16((size_t)(s->ctx + 64) / 64 * 64 * 4);
    if (a.v_off + att_bytes + 16 > dyn) return persist_no("the context's keys do not fit shared memory");
    a.vcap0 = (int)((dyn - a.v_off - att_bytes - 16) / ((size_t)hd * es));
    a.att_off = al16(a.v_off + (size_t)a.vcap0 * hd * es);
    if (a.att_off + att_bytes > dyn) return persist_no("the attention shared-memory plan does not fit");
    // every CTA resident at once (one per SM)
    int occ = 0;
    if (s->kv_fp16) {
        CK(cudaFuncSetAttribute(ember_persist_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
        CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ember_persist_kernel<__half>, PTT, dyn));
    } else {
        CK(cudaFuncSetAttribute(ember_persist_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
        CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ember_persist_kernel<float>, PTT, dyn));
    }
    int coop = 0;
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device));
    if (occ < 1 || !coop) return persist_no("no cooperative launch of one CTA per SM");
    // per-layer pointers
    std::vector<PLayer> hl(m->n_layers);
    for (int l = 0; l < m->n_layers; l++) {
        const DevLayer &L = m->layers[l];
        const DevMat *ms[7] = {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3};
        for (int k = 0; k < 7; k++) { hl[l].q[k] = ms[k]->q; hl[l].s[k] = ms[k]->s; }
        hl[l].attn_norm = L.attn_norm; hl[l].ffn_norm = L.ffn_norm; hl[l].q_norm = L.q_norm; hl[l].k_norm = L.k_norm;
        hl[l].bq = L.bq; hl[l].bk = L.bk; hl[l].bv = L.bv;
    }
    PLayer *dl = nullptr;
    if (salloc(s, (void **)&dl, hl.size() * sizeof(PLayer))) return 1;
    CK(cudaMemcpy(dl, hl.data(), hl.size() * sizeof(PLayer), cudaMemcpyHostToDevice));
    a.layers = dl;
    a.has_bias = m->layers[0].bq != nullptr;
    // hand-off words, zero (no tag matches 0)
    const size_t nqkv = qd + 2 * kvd, no = qd / 4 + qd / 32, nx = 2 * (size_t)m->dim;
    const size_t nh = m->hidden / 4 + m->hidden / 32, nam = 2 * (size_t)G;
    PState *ps = new PState();
    ps->words_bytes = (nqkv + no + nx + nh + nam) * 8;
    if (salloc(s, (void **)&ps->words, ps->words_bytes)) { delete ps; return 1; }
    a.w_qkv = ps->words;
    a.w_o = a.w_qkv + nqkv;
    a.w_x = a.w_o + no;
    a.w_h = a.w_x + nx;
    a.w_am = a.w_h + nh;
    if (cudaMemset(ps->words, 0, ps->words_bytes) != cudaSuccess) { delete ps; return set_err("hand-off buffer init failed"); }
    ps->a = a;
    ps->smem = dyn;
    ps->grid = m->n_sm;
    ps->tag = 1;
    ps->tag_stride = 8u * (uint32_t)m->n_layers + 8u;
    int one = 1;
    if (cudaMemcpy(s->ctl + CTL_TAG, &one, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
        delete ps;
        return set_err("hand-off tag init failed");
    }
    s->ps = ps;
    g_persist_why[0] = 0;
    return 0;
}

void emb::persist_release(EmberCudaState *s) {
    delete s->ps;
    s->ps = nullptr;
}

// Enqueue one launch on the state's stream: n_steps token steps starting from
// ctl's token and position (greedy picks between steps and the picked tokens
// to out_tokens when greedy; one forward step otherwise).
int emb::persist_run(EmberCudaState *s, int n_steps, int greedy) {
    PState *ps = s->ps;
    // tags are 32-bit: before they could wrap, clear the words and start over
    const uint64_t need = (uint64_t)ps->tag + (uint64_t)n_steps * ps->tag_stride;
    if (need >= 0x7FFFFFFFull) {
        CK(cudaMemsetAsync(ps->words, 0, ps->words_bytes, s->stream));
        ps->tag = 1;
        CK(cudaMemcpyAsync(s->ctl + CTL_TAG, &ps->tag, sizeof(int), cudaMemcpyHostToDevice, s->stream));
        CK(cudaStreamSynchronize(s->stream));
    }
    PArgs a = ps->a;
    a.n_steps = n_steps;
    a.out_tokens = greedy ? s->out_tokens : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ps->grid);
    cfg.blockDim = dim3((unsigned)PTT);
    cfg.dynamicSmemBytes = ps->smem;
    cfg.stream = s->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (s->kv_fp16) CK(cudaLaunchKernelEx(&cfg, ember_persist_kernel<__half>, a));
    else CK(cudaLaunchKernelEx(&cfg, ember_persist_kernel<float>, a));
    ps->tag += (uint32_t)n_steps * ps->tag_stride;
    return 0;
}

#ifdef EMBER_PROBES
// profiling build only: the phase timestamps of the last launch
extern "C" int ember_cuda_pprobe_read(unsigned long long *out) {
    if (cudaDeviceSynchronize() != cudaSuccess) return 1;
    return cudaMemcpyFromSymbol(out, g_pp, sizeof(g_pp)) != cudaSuccess;
}
#endif
