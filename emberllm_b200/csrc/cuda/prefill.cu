// prefill.cu — host side of the batched prefill (ref src/model.c:283-360) and of
// the op-level ember_matmul_batch (ref src/kernels.c:227-264).
//
// Weight packs. The first batched prefill on a model builds, per layer, four
// int8 matrices in the layout the tensor-core GEMM reads through TMA: q|k|v rows
// concatenated (one GEMM), wo, w1|w3 concatenated (one GEMM, SwiGLU reads both
// halves of a row), w2. Rows are padded to a multiple of 128 and K to a multiple
// of 128 bytes (zeros), Q4_0 nibbles are expanded to int8 (q - 8), and the
// block scales are widened to fp32 rows [rows_pad][nbp]. The packs are a second
// copy of the layer weights (the decode path keeps the compact Q8_0 / Q4_0 rows).
//
// Activations. A state's prefill scratch holds PF_CHUNK tokens: the residual
// stream X [n][dim], the int8 GEMM input XQ [n_pad][k_pad] with its block scales
// XS [nb][n_pad], the q|k|v output, the roped queries and the w1|w3 output.
// Longer prompts run in chunks of PF_CHUNK tokens (the per-token arithmetic does
// not depend on how tokens are grouped).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "ember_ops.h"
#include "prefill_kernels.cuh"
#include "runtime_internal.cuh"

namespace emb {

constexpr int PF_CHUNK = 512;              // tokens per batched pass
// token-tile widths of the GEMM: BN = 16 runs three CTAs per SM, 32 and 64 two,
// 128 one (the last is the 128-row box the swapped GEMM reads its A operand with)
constexpr int PF_NBN = 4;
constexpr int PF_BNS[PF_NBN] = { 16, 32, 64, 128 };

static size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

// ------------------------------------------------------------ tensor maps ----

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// an int8 matrix [outer][inner] (row stride = inner bytes) read in boxes of
// 128 bytes x box_rows rows with 128-byte swizzle
static int map_i8(CUtensorMap *map, const void *base, size_t inner, size_t outer, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_err("cuTensorMapEncodeTiled is not available from the driver");
    if (inner % 128 || (uintptr_t)base % 16) return set_err("tensor map: unaligned int8 matrix");
    cuuint64_t dims[2] = { (cuuint64_t)inner, (cuuint64_t)outer };
    cuuint64_t strides[1] = { (cuuint64_t)inner };
    cuuint32_t box[2] = { 128u, (cuuint32_t)box_rows };
    cuuint32_t es[2] = { 1u, 1u };
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// a 2-D fp32 / fp16 matrix [outer][inner] (row stride = inner elements), boxes
// of box_inner x box_outer elements, no swizzle
int map_2d(CUtensorMap *map, const void *base, int elem_bytes, size_t inner, size_t outer, int box_inner,
           int box_outer) {
    auto fn = encode_fn();
    if (!fn) return set_err("cuTensorMapEncodeTiled is not available from the driver");
    if ((inner * elem_bytes) % 16 || (box_inner * elem_bytes) % 16 || (uintptr_t)base % 16)
        return set_err("tensor map: unaligned matrix");
    cuuint64_t dims[2] = { (cuuint64_t)inner, (cuuint64_t)outer };
    cuuint64_t strides[1] = { (cuuint64_t)inner * elem_bytes };
    cuuint32_t box[2] = { (cuuint32_t)box_inner, (cuuint32_t)box_outer };
    cuuint32_t es[2] = { 1u, 1u };
    CUresult r = fn(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

// ------------------------------------------------------------ kernel setup ---

template <typename K>
static int pf_allow_smem(K kernel, int bytes) {
    CK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return 0;
}

static int g_att_smem_cap = 0;   // dynamic smem the attention kernel may use
static int g_mtv_smem_cap = 0;   // dynamic smem the multi-token GEMV may use

static int pf_init(int device) {
    static unsigned done = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 32 && ((done >> device) & 1u)) return 0;
    int optin = 0;
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    if (pf_allow_smem(pf_gemm_kernel<PF_SW_BN, PF_EPI_STORE, true>, PfLayout<PF_SW_BN>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<PF_SW_BN, PF_EPI_RESID, true>, PfLayout<PF_SW_BN>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<16, PF_EPI_STORE>, PfLayout<16>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<16, PF_EPI_RESID>, PfLayout<16>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<32, PF_EPI_STORE>, PfLayout<32>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<32, PF_EPI_RESID>, PfLayout<32>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<64, PF_EPI_STORE>, PfLayout<64>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<64, PF_EPI_RESID>, PfLayout<64>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<128, PF_EPI_STORE>, PfLayout<128>::SMEM) ||
        pf_allow_smem(pf_gemm_kernel<128, PF_EPI_RESID>, PfLayout<128>::SMEM))
        return 1;
    // one cap for every attention instantiation (the largest static shared memory)
    int cap = optin;
    auto cap_of = [&](const void *k) {
        cudaFuncAttributes f;
        if (cudaFuncGetAttributes(&f, k) == cudaSuccess && optin - (int)f.sharedSizeBytes < cap)
            cap = optin - (int)f.sharedSizeBytes;
    };
#define EMB_PF_ATT_EACH(X)                                                                                   \
    X(float, 4, 4) X(float, 8, 4) X(float, 8, 8) X(float, 16, 4) X(float, 16, 8) X(float, 16, 16)            \
    X(__half, 4, 4) X(__half, 8, 4) X(__half, 8, 8) X(__half, 16, 4) X(__half, 16, 8) X(__half, 16, 16)      \
    X(float, 4, 8) X(float, 4, 16) X(float, 8, 16) X(__half, 4, 8) X(__half, 4, 16) X(__half, 8, 16)
#define EMB_CAP(T, RS, RG) cap_of((const void *)pf_attn_kernel<T, RS, RG>);
    EMB_PF_ATT_EACH(EMB_CAP)
#undef EMB_CAP
#define EMB_ALLOW(T, RS, RG) if (pf_allow_smem(pf_attn_kernel<T, RS, RG>, cap)) return 1;
    EMB_PF_ATT_EACH(EMB_ALLOW)
#undef EMB_ALLOW
#undef EMB_PF_ATT_EACH
    g_att_smem_cap = cap;
    // the multi-token GEMV
    cudaFuncAttributes fa;
    {
        CK(cudaFuncGetAttributes(&fa, pf_mtv_kernel<PF_EPI_STORE>));
        const int c1 = optin - (int)fa.sharedSizeBytes;
        CK(cudaFuncGetAttributes(&fa, pf_mtv_kernel<PF_EPI_RESID>));
        const int c2 = optin - (int)fa.sharedSizeBytes;
        g_mtv_smem_cap = c1 < c2 ? c1 : c2;
        if (pf_allow_smem(pf_mtv_kernel<PF_EPI_STORE>, g_mtv_smem_cap) ||
            pf_allow_smem(pf_mtv_kernel<PF_EPI_RESID>, g_mtv_smem_cap))
            return 1;
    }
    // the batched decode attention (attn_decode_kernel, BATCH mode)
    CK(cudaFuncGetAttributes(&fa, attn_decode_kernel<float, true>));
    if (pf_allow_smem(attn_decode_kernel<float, true>, optin - (int)fa.sharedSizeBytes)) return 1;
    CK(cudaFuncGetAttributes(&fa, attn_decode_kernel<__half, true>));
    if (pf_allow_smem(attn_decode_kernel<__half, true>, optin - (int)fa.sharedSizeBytes)) return 1;
#define EMB_AB_ALLOW(T, K)                                                                    \
    CK(cudaFuncGetAttributes(&fa, attn_batch_kernel<T, K>));                                  \
    if (pf_allow_smem(attn_batch_kernel<T, K>, optin - (int)fa.sharedSizeBytes)) return 1;
    EMB_AB_ALLOW(float, 1) EMB_AB_ALLOW(float, 2) EMB_AB_ALLOW(float, 3) EMB_AB_ALLOW(float, 4)
    EMB_AB_ALLOW(__half, 1) EMB_AB_ALLOW(__half, 2) EMB_AB_ALLOW(__half, 3) EMB_AB_ALLOW(__half, 4)
#undef EMB_AB_ALLOW
    if (device < 32) done |= 1u << device;
    return 0;
}

// ------------------------------------------------------------ weight packs ---

struct PfMat {
    int8_t *q = nullptr;
    float *s = nullptr;
    float *s_t = nullptr;      // the scales transposed, [nbp][rows_pad] (swapped GEMM)
    int rows = 0, rows_pad = 0, k = 0, k_pad = 0, nb = 0, nbp = 0;
    CUtensorMap map;           // A operand: boxes of 128 rows x 128 bytes
    CUtensorMap map_sw;        // B operand of the swapped GEMM: boxes of PF_SW_BN rows
};

struct PfLayerPack {
    PfMat qkv, wo, w13, w2;
};

struct PfModel {
    std::vector<PfLayerPack> layers;
    PfMat head;                // lm_head, for batched decode (built on first use)
    int head_ready = 0;
    std::vector<void *> allocs;
};

static int pf_alloc(std::vector<void *> &v, void **p, size_t n) {
    CK(cudaMalloc(p, n ? n : 16));
    v.push_back(*p);
    return 0;
}

// concatenate the row blocks of `parts` (same cols, quantized) into one pack
static int build_pack(PfModel *pm, PfMat *pk, const DevMat *const *parts, int nparts) {
    const int k = parts[0]->cols;
    int rows = 0;
    for (int i = 0; i < nparts; i++) {
        if (parts[i]->cols != k || parts[i]->dtype == EMBER_DT_F32) return set_err("prefill pack: bad matrix");
        rows += parts[i]->rows;
    }
    pk->rows = rows;
    pk->rows_pad = (int)round_up((size_t)rows, PF_BM);
    pk->k = k;
    pk->k_pad = (int)round_up((size_t)k, PF_BK);
    pk->nb = k / 32;
    pk->nbp = (int)round_up((size_t)pk->nb, 4);
    const size_t qbytes = (size_t)pk->rows_pad * pk->k_pad, sbytes = (size_t)pk->rows_pad * pk->nbp * 4;
    if (pf_alloc(pm->allocs, (void **)&pk->q, qbytes) || pf_alloc(pm->allocs, (void **)&pk->s, sbytes) ||
        pf_alloc(pm->allocs, (void **)&pk->s_t, sbytes))
        return 1;
    CK(cudaMemset(pk->q, 0, qbytes));
    CK(cudaMemset(pk->s, 0, sbytes));
    int r0 = 0;
    for (int i = 0; i < nparts; i++) {
        PfPackArgs a;
        a.q = parts[i]->q; a.s = parts[i]->s; a.dtype = parts[i]->dtype; a.rows = parts[i]->rows; a.nb = pk->nb;
        a.dq = pk->q + (size_t)r0 * pk->k_pad; a.ds = pk->s + (size_t)r0 * pk->nbp;
        a.k_pad = pk->k_pad; a.nbp = pk->nbp;
        const long long total = (long long)a.rows * a.nb;
        const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
        pf_pack_kernel<<<grid > 0 ? grid : 1, 256>>>(a);
        CK(cudaGetLastError());
        r0 += parts[i]->rows;
    }
    {
        const long long total = (long long)pk->rows_pad * pk->nbp;
        const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
        pf_transpose_kernel<<<grid, 256>>>(pk->s, pk->s_t, pk->rows_pad, pk->nbp);
        CK(cudaGetLastError());
    }
    return map_i8(&pk->map, pk->q, (size_t)pk->k_pad, (size_t)pk->rows_pad, PF_BM) ||
           map_i8(&pk->map_sw, pk->q, (size_t)pk->k_pad, (size_t)pk->rows_pad, PF_SW_BN);
}

int pf_supported(const EmberCudaModel *m) {
    if (m->head_dim > 256 || m->head_dim % 32) return 0;
    if (m->n_heads / m->n_kv > PF_ATT_MAX_ROWS) return 0;
    for (const DevLayer &L : m->layers) {
        const DevMat *mats[7] = { &L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3 };
        for (const DevMat *d : mats)
            if (d->dtype != EMBER_DT_Q8_0 && d->dtype != EMBER_DT_Q4_0) return 0;
    }
    return 1;
}

static int pf_prepare_model(EmberCudaModel *m) {
    if (m->pf) return 0;
    if (pf_init(m->device)) return 1;
    PfModel *pm = new PfModel();
    pm->layers.resize(m->layers.size());
    int rc = 0;
    for (size_t l = 0; l < m->layers.size() && !rc; l++) {
        const DevLayer &L = m->layers[l];
        PfLayerPack &P = pm->layers[l];
        const DevMat *qkv[3] = { &L.wq, &L.wk, &L.wv };
        const DevMat *wo[1] = { &L.wo };
        const DevMat *w13[2] = { &L.w1, &L.w3 };
        const DevMat *w2[1] = { &L.w2 };
        rc = build_pack(pm, &P.qkv, qkv, 3) || build_pack(pm, &P.wo, wo, 1) || build_pack(pm, &P.w13, w13, 2) ||
             build_pack(pm, &P.w2, w2, 1);
    }
    if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = set_err("prefill pack build failed");
    if (rc) {
        for (void *p : pm->allocs) cudaFree(p);
        delete pm;
        return 1;
    }
    m->pf = pm;
    return 0;
}

void pf_model_release(EmberCudaModel *m) {
    if (!m || !m->pf) return;
    for (void *p : m->pf->allocs) cudaFree(p);
    delete m->pf;
    m->pf = nullptr;
}

// ------------------------------------------------------------ state scratch --

enum { PF_K_DIM = 0, PF_K_QD = 1, PF_K_HID = 2 };

struct PfState {
    int n_cap = 0, n_pad = 0;
    int k_pad[3] = { 0, 0, 0 };
    float *X = nullptr, *XS = nullptr, *QKV = nullptr, *QR = nullptr, *H = nullptr;
    int8_t *XQ = nullptr;
    int ld_qkv = 0, ld_h = 0;
    CUtensorMap mapB[3][PF_NBN];    // [K kind][BN index]
    std::vector<void *> allocs;
};

// activations for up to n_cap token rows
static int pf_state_new(EmberCudaModel *m, int n_cap, PfState **out) {
    PfState *ps = new PfState();
    const int hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
    ps->n_cap = n_cap;
    ps->n_pad = (int)round_up((size_t)n_cap, 128);
    const int ks[3] = { m->dim, qd, m->hidden };
    size_t kmax = 0;
    int nbmax = 0;
    for (int i = 0; i < 3; i++) {
        ps->k_pad[i] = (int)round_up((size_t)ks[i], PF_BK);
        if ((size_t)ps->k_pad[i] > kmax) kmax = ps->k_pad[i];
        if (ks[i] / 32 > nbmax) nbmax = ks[i] / 32;
    }
    const PfLayerPack &P0 = m->pf->layers[0];
    ps->ld_qkv = P0.qkv.rows_pad;
    ps->ld_h = P0.w13.rows_pad;
    (void)kvd;
    int rc = pf_alloc(ps->allocs, (void **)&ps->X, (size_t)ps->n_cap * m->dim * 4) ||
             pf_alloc(ps->allocs, (void **)&ps->XQ, (size_t)ps->n_pad * kmax) ||
             pf_alloc(ps->allocs, (void **)&ps->XS, (size_t)nbmax * ps->n_pad * 4) ||
             pf_alloc(ps->allocs, (void **)&ps->QKV, (size_t)ps->n_cap * ps->ld_qkv * 4) ||
             pf_alloc(ps->allocs, (void **)&ps->QR, (size_t)ps->n_cap * qd * 4) ||
             pf_alloc(ps->allocs, (void **)&ps->H, (size_t)ps->n_cap * ps->ld_h * 4);
    if (!rc && (cudaMemset(ps->XQ, 0, (size_t)ps->n_pad * kmax) != cudaSuccess ||
                cudaMemset(ps->XS, 0, (size_t)nbmax * ps->n_pad * 4) != cudaSuccess))
        rc = set_err("prefill scratch initialisation failed");
    for (int i = 0; i < 3 && !rc; i++)
        for (int j = 0; j < PF_NBN && !rc; j++)
            rc = map_i8(&ps->mapB[i][j], ps->XQ, (size_t)ps->k_pad[i], (size_t)ps->n_pad, PF_BNS[j]);
    if (rc) {
        for (void *p : ps->allocs) cudaFree(p);
        delete ps;
        return 1;
    }
    *out = ps;
    return 0;
}

static void pf_state_free(PfState *ps) {
    if (!ps) return;
    for (void *p : ps->allocs) cudaFree(p);
    delete ps;
}

static int pf_prepare_state(EmberCudaState *s) {
    if (s->pf) return 0;
    return pf_state_new(s->m, PF_CHUNK, &s->pf);
}

void pf_state_release(EmberCudaState *s) {
    if (!s || !s->pf) return;
    for (void *p : s->pf->allocs) cudaFree(p);
    delete s->pf;
    s->pf = nullptr;
}

// ------------------------------------------------------------ launches -------

// Token-tile width: the one that minimises the busiest SM's share of the
// epilogue's fp32 work (tiles per SM x width); ties go to the narrow tile,
// which spreads over more SMs and runs two CTAs per SM.
static int choose_bn(int rows_pad, int n, int n_sm) {
    const char *force = getenv("EMBER_PF_BN");      // tuning: force a width
    if (force && *force)
        for (int j = 0; j < PF_NBN; j++)
            if (atoi(force) == PF_BNS[j]) return j;
    int best = 0;
    long long best_cost = -1;
    for (int j = 0; j < PF_NBN; j++) {
        const int bn = PF_BNS[j];
        const long long tiles = (long long)(rows_pad / PF_BM) * ((n + bn - 1) / bn);
        const long long cost = (tiles + n_sm - 1) / n_sm * bn;
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = j; }
    }
    return best;
}

// swapped operands (few tokens): A = the activations' 128-row box, B = PF_SW_BN
// weight rows; one CTA per (token tile, PF_SW_BN weight rows)
template <int EPI>
static int launch_gemm_sw(const PfMat &w, const CUtensorMap &ma, const PfGemmArgs &a, cudaStream_t st) {
    dim3 grid((unsigned)(a.n_pad / PF_BM), (unsigned)(w.rows_pad / PF_SW_BN));
    pf_gemm_kernel<PF_SW_BN, EPI, true><<<grid, PfLayout<PF_SW_BN>::THREADS, PfLayout<PF_SW_BN>::SMEM, st>>>(
        ma, w.map_sw, a);
    CK(cudaGetLastError());
    return 0;
}

// Swapped operands, opt-in (EMBER_PF_SWAP=1): for few tokens it spreads a
// matrix over rows_pad/PF_SW_BN CTAs instead of rows_pad/128, but each CTA's
// epilogue walks as many (row, token) chains as before, so it measured slower
// (16 streams: 3.70k vs 3.95k tok/s; 32: 6.98k vs 7.26k); taken, when asked,
// where the usual tiling leaves most SMs idle.
static bool use_swap(int rows_pad, int n, int n_pad, int n_sm) {
    const char *f = getenv("EMBER_PF_SWAP");
    if (!(f && atoi(f) != 0)) return false;
    const long long plain = (long long)(rows_pad / PF_BM) * ((n + 31) / 32);
    const long long sw = (long long)(rows_pad / PF_SW_BN) * (n_pad / PF_BM);
    return plain < n_sm && sw > plain;
}

template <int BN, int EPI>
static int launch_gemm_bn(const PfMat &w, const CUtensorMap &mb, const PfGemmArgs &a, cudaStream_t st) {
    dim3 grid((unsigned)(w.rows_pad / PF_BM), (unsigned)((a.n + BN - 1) / BN));
    pf_gemm_kernel<BN, EPI><<<grid, PfLayout<BN>::THREADS, PfLayout<BN>::SMEM, st>>>(w.map, mb, a);
    CK(cudaGetLastError());
    return 0;
}

// Few tokens: the dp4a multi-token GEMV. It wins on the short, long-K residual
// matrices (wo, w2: a tensor-core CTA walks 64-96 serial block MMAs) up to 64
// tokens, on the others only up to 16 (Qwen3 streams, measured: 16 streams 4.8k ->
// 6.7k tok/s; 32 streams best without it on q|k|v and w1|w3; 64 streams 14.7k ->
// 17.1k), and never on the vocabulary-sized head. EMBER_PF_MTV sets the first
// count (0 disables it), EMBER_PF_MTV_STORE the second (tuning).
static bool use_mtv(int n, bool resid, int rows) {
    static int cap = -1, cap_store = -1;
    if (cap < 0) {
        const char *e = getenv("EMBER_PF_MTV");
        cap = e && *e ? atoi(e) : 64;
        if (cap < 0) cap = 0;
        const char *f = getenv("EMBER_PF_MTV_STORE");
        cap_store = f && *f ? atoi(f) : 16;
        if (cap_store > cap) cap_store = cap;
    }
    if (rows > 16384) return false;
    return n <= (resid ? cap : cap_store);
}

template <int EPI>
static int launch_mtv(const PfMat &w, const int8_t *xq, const float *xs, int n_pad, int n, float *out, int ld,
                      int *err, cudaStream_t st) {
    PfMtvArgs a;
    a.wq = w.q; a.ws = w.s; a.xq = xq; a.xs = xs; a.out = out; a.err = err;
    a.rows = w.rows; a.nb = w.nb; a.nbp = w.nbp; a.k_pad = w.k_pad; a.n = n; a.n_pad = n_pad; a.ld = ld;
    const size_t sm = mtv_smem_bytes(w.k_pad, w.nbp);
    dim3 grid((unsigned)(w.rows_pad / MTV_R), (unsigned)((n + MTV_T - 1) / MTV_T));
    pf_mtv_kernel<EPI><<<grid, MTV_R * MTV_T, sm, st>>>(a);
    CK(cudaGetLastError());
    return 0;
}

static int launch_gemm(const PfMat &w, const CUtensorMap (&maps)[PF_NBN], const int8_t *xq, const float *xs,
                       int n_pad, int n, float *out, int ld, bool resid, int *err, int n_sm, cudaStream_t st) {
    if (xq && use_mtv(n, resid, w.rows) && mtv_smem_bytes(w.k_pad, w.nbp) <= (size_t)g_mtv_smem_cap)
        return resid ? launch_mtv<PF_EPI_RESID>(w, xq, xs, n_pad, n, out, ld, err, st)
                     : launch_mtv<PF_EPI_STORE>(w, xq, xs, n_pad, n, out, ld, err, st);
    PfGemmArgs a;
    a.ws = w.s; a.ws_t = w.s_t; a.rows_pad = w.rows_pad; a.xs = xs; a.out = out; a.err = err;
    a.rows = w.rows; a.nb = w.nb; a.nbp = w.nbp; a.n = n; a.n_pad = n_pad; a.ld = ld;
    if (use_swap(w.rows_pad, n, n_pad, n_sm)) {
        // the activations' 128-row box map (PF_BNS[PF_NBN - 1] == PF_BM)
        return resid ? launch_gemm_sw<PF_EPI_RESID>(w, maps[PF_NBN - 1], a, st)
                     : launch_gemm_sw<PF_EPI_STORE>(w, maps[PF_NBN - 1], a, st);
    }
    const int j = choose_bn(w.rows_pad, n, n_sm);
    switch (j * 2 + (resid ? 1 : 0)) {
    case 0: return launch_gemm_bn<16, PF_EPI_STORE>(w, maps[0], a, st);
    case 1: return launch_gemm_bn<16, PF_EPI_RESID>(w, maps[0], a, st);
    case 2: return launch_gemm_bn<32, PF_EPI_STORE>(w, maps[1], a, st);
    case 3: return launch_gemm_bn<32, PF_EPI_RESID>(w, maps[1], a, st);
    case 4: return launch_gemm_bn<64, PF_EPI_STORE>(w, maps[2], a, st);
    case 5: return launch_gemm_bn<64, PF_EPI_RESID>(w, maps[2], a, st);
    case 6: return launch_gemm_bn<128, PF_EPI_STORE>(w, maps[3], a, st);
    default: return launch_gemm_bn<128, PF_EPI_RESID>(w, maps[3], a, st);
    }
}

// attention tile: the most tokens per CTA (rows = tokens x kv_mul <= 16 at
// head_dim 128, <= 8 at head_dim 64 and below, where the shorter chains favour
// more, smaller CTAs -- measured: SmolLM2 pp512 96k -> 105k tok/s, Qwen3 best at
// 16; EMBER_PF_ATT_ROWS overrides, a tuning knob) whose weights [positions][rows
// rounded up to 4] fit shared memory; 0 if none does
static int attn_tile(const EmberCudaModel *m, int p_cap, int *tq, int *rs) {
    const int kv_mul = m->n_heads / m->n_kv;
    const char *rc = getenv("EMBER_PF_ATT_ROWS");
    const int def_rows = m->head_dim <= 64 && kv_mul <= 8 ? 8 : PF_ATT_MAX_ROWS;
    const int max_rows = rc && atoi(rc) >= kv_mul && atoi(rc) <= PF_ATT_MAX_ROWS ? atoi(rc) : def_rows;
    for (int t = max_rows / kv_mul; t > 0; t--) {
        const int r = (t * kv_mul + 3) / 4 * 4;
        if (pf_attn_smem(p_cap, r, m->head_dim, 4) <= (size_t)g_att_smem_cap) {   // fp32 cache: the larger
            *tq = t;
            *rs = r;
            return 1;
        }
    }
    return 0;
}

int pf_fits(EmberCudaState *s, int n, int start) {
    if (pf_init(s->m->device)) return 0;
    int tq, rs;
    return attn_tile(s->m, (int)round_up((size_t)(start + n), 4), &tq, &rs);
}

// The rows' positions and where their keys and values go: consecutive
// positions start.. in one cache (prefill), or each row its own position pos[t]
// and its own cache at kc/vc + t * cache_stride (batched decode of streams).
struct PfSeq {
    int n, start;
    const int *pos;
    size_t cache_stride;             // elements
    void *kc, *vc;                   // layer-0 cache of row 0
    size_t k_layer, v_layer;         // elements per layer
    int ctx, kstride, kv_fp16;
    const float2 *rope;
    int tq, rs, p_cap;               // attention tiling
    // batched decode: attention as the single-token kernel, one CTA per (query
    // head, stream), with this chunking and shared memory (scores in shared memory)
    int dec_attn, dec_chunk;
    size_t dec_smem;
    int *ctl;                        // error word
};

// the attention instantiation for (cache type, register rows, output rows)
template <typename T, int RS>
static void launch_pf_attn_rs(int rg, dim3 grid, size_t smem, cudaStream_t st, const PfAttnArgs &aa) {
    if (rg <= 4) pf_attn_kernel<T, RS, 4><<<grid, PF_ATT_THREADS, smem, st>>>(aa);
    else if (rg <= 8) pf_attn_kernel<T, RS, 8><<<grid, PF_ATT_THREADS, smem, st>>>(aa);
    else pf_attn_kernel<T, RS, 16><<<grid, PF_ATT_THREADS, smem, st>>>(aa);
}
static int launch_pf_attn(bool fp16, int rs, int rg, dim3 grid, size_t smem, cudaStream_t st, const PfAttnArgs &aa) {
    if (rs <= 4) {
        if (fp16) launch_pf_attn_rs<__half, 4>(rg, grid, smem, st, aa);
        else launch_pf_attn_rs<float, 4>(rg, grid, smem, st, aa);
    } else if (rs <= 8) {
        if (fp16) launch_pf_attn_rs<__half, 8>(rg, grid, smem, st, aa);
        else launch_pf_attn_rs<float, 8>(rg, grid, smem, st, aa);
    } else {
        if (fp16) launch_pf_attn_rs<__half, 16>(rg, grid, smem, st, aa);
        else launch_pf_attn_rs<float, 16>(rg, grid, smem, st, aa);
    }
    CK(cudaGetLastError());
    return 0;
}

// embedding + every layer for q.n token rows of ids_dev, on ps->X
static int pf_layers(EmberCudaModel *m, PfState *ps, const PfSeq &q, const int *ids_dev, int *err, cudaStream_t st) {
    const int nc = q.n, hd = m->head_dim;
    const size_t es = q.kv_fp16 ? 2 : 4;
    {
        PfEmbedArgs ea;
        ea.q = m->tok_emb.q; ea.s = m->tok_emb.s; ea.dtype = m->tok_emb.dtype; ea.dim = m->dim;
        ea.vocab = m->vocab; ea.ids = ids_dev; ea.x = ps->X; ea.err = err;
        pf_embed_kernel<<<nc, 256, 0, st>>>(ea);
        CK(cudaGetLastError());
    }
    for (int l = 0; l < m->n_layers; l++) {
        const DevLayer &L = m->layers[l];
        const PfLayerPack &P = m->pf->layers[l];
        PfTokArgs ta;
        memset(&ta, 0, sizeof(ta));
        ta.xq = ps->XQ; ta.xs = ps->XS; ta.n_pad = ps->n_pad; ta.ex = m->ex; ta.eps = m->eps;
        // attention block
        ta.x = ps->X; ta.ld_x = m->dim; ta.norm_w = L.attn_norm; ta.cols = m->dim; ta.k_pad = ps->k_pad[PF_K_DIM];
        pf_norm_quant_kernel<<<nc, 256, (size_t)m->dim * 8, st>>>(ta);
        CK(cudaGetLastError());
        if (launch_gemm(P.qkv, ps->mapB[PF_K_DIM], ps->XQ, ps->XS, ps->n_pad, nc, ps->QKV, ps->ld_qkv, false, err, m->n_sm, st))
            return 1;
        PfQkvArgs qa;
        qa.qkv = ps->QKV; qa.ld = ps->ld_qkv; qa.bq = L.bq; qa.bk = L.bk; qa.bv = L.bv;
        qa.q_norm = m->qk_norm ? L.q_norm : nullptr; qa.k_norm = m->qk_norm ? L.k_norm : nullptr;
        qa.rope = q.rope; qa.qr = ps->QR;
        qa.kc = (char *)q.kc + (size_t)l * q.k_layer * es;
        qa.vc = (char *)q.vc + (size_t)l * q.v_layer * es;
        qa.nh = m->n_heads; qa.nkv = m->n_kv; qa.hd = hd; qa.ctx = q.ctx; qa.kstride = q.kstride;
        qa.neox = m->rope_neox; qa.start = q.start; qa.pos = q.pos; qa.cache_stride = q.cache_stride; qa.eps = m->eps;
        qa.n = nc;
        const unsigned qgrid = (unsigned)((nc * (m->n_heads + m->n_kv) + PF_QKV_WARPS - 1) / PF_QKV_WARPS);
        if (q.kv_fp16) pf_qkv_post_kernel<__half><<<qgrid, 32 * PF_QKV_WARPS, 0, st>>>(qa);
        else pf_qkv_post_kernel<float><<<qgrid, 32 * PF_QKV_WARPS, 0, st>>>(qa);
        CK(cudaGetLastError());
        PfAttnArgs aa;
        aa.qr = ps->QR; aa.kc = qa.kc; aa.vc = qa.vc; aa.xq = ps->XQ; aa.k_pad = ps->k_pad[PF_K_QD];
        aa.xs = ps->XS; aa.n_pad = ps->n_pad; aa.nh = m->n_heads; aa.nkv = m->n_kv; aa.hd = hd;
        aa.ctx = q.ctx; aa.kstride = q.kstride; aa.start = q.start; aa.n = nc; aa.tq = q.tq; aa.rs = q.rs;
        aa.p_cap = q.p_cap; aa.pos = q.pos; aa.cache_stride = q.cache_stride; aa.ex = m->ex;
        const dim3 agrid((unsigned)m->n_kv, (unsigned)((nc + q.tq - 1) / q.tq));
        const size_t asmem = pf_attn_smem(q.p_cap, q.rs, hd, (int)es);
        if (q.dec_attn) {
            AttnArgs da;
            memset(&da, 0, sizeof(da));
            da.q = ps->QR; da.kc = qa.kc; da.vc = qa.vc; da.ctl = q.ctl;
            da.nh = m->n_heads; da.nkv = m->n_kv; da.hd = hd; da.ctx = q.ctx; da.kstride = q.kstride;
            da.att_in_smem = 1; da.chunk = q.dec_chunk; da.ex = m->ex;
            da.bpos = q.pos; da.cache_stride = q.cache_stride;
            da.bxq = ps->XQ; da.bxs = ps->XS; da.k_pad = ps->k_pad[PF_K_QD]; da.n_pad = ps->n_pad;
            const int kvm = m->n_heads / m->n_kv;
            if (q.dec_attn == 1 && kvm <= 4 && kvm * hd <= ATTN_THREADS) {
                // one CTA per (kv head, stream): its query heads share each staged chunk
                const dim3 bgrid((unsigned)m->n_kv, (unsigned)nc);
                const size_t bsm = ab_smem_bytes(hd, (int)es, kvm, q.ctx);
#define EMB_AB(T)                                                                                   \
    switch (kvm) {                                                                                  \
    case 1: attn_batch_kernel<T, 1><<<bgrid, ATTN_THREADS, bsm, st>>>(da); break;                    \
    case 2: attn_batch_kernel<T, 2><<<bgrid, ATTN_THREADS, bsm, st>>>(da); break;                    \
    case 3: attn_batch_kernel<T, 3><<<bgrid, ATTN_THREADS, bsm, st>>>(da); break;                    \
    default: attn_batch_kernel<T, 4><<<bgrid, ATTN_THREADS, bsm, st>>>(da); break;                   \
    }
                if (q.kv_fp16) { EMB_AB(__half) } else { EMB_AB(float) }
#undef EMB_AB
            } else {
                const dim3 dgrid((unsigned)m->n_heads, (unsigned)nc);
                if (q.kv_fp16) attn_decode_kernel<__half, true><<<dgrid, ATTN_THREADS, q.dec_smem, st>>>(da);
                else attn_decode_kernel<float, true><<<dgrid, ATTN_THREADS, q.dec_smem, st>>>(da);
            }
        } else {
            if (launch_pf_attn(q.kv_fp16 != 0, q.rs, pf_attn_rows_per_group(q.rs, hd), agrid, asmem, st, aa)) return 1;
        }
        CK(cudaGetLastError());
        if (launch_gemm(P.wo, ps->mapB[PF_K_QD], ps->XQ, ps->XS, ps->n_pad, nc, ps->X, m->dim, true, err, m->n_sm, st))
            return 1;
        // feed-forward block
        ta.x = ps->X; ta.ld_x = m->dim; ta.norm_w = L.ffn_norm; ta.cols = m->dim; ta.k_pad = ps->k_pad[PF_K_DIM];
        pf_norm_quant_kernel<<<nc, 256, (size_t)m->dim * 8, st>>>(ta);
        CK(cudaGetLastError());
        if (launch_gemm(P.w13, ps->mapB[PF_K_DIM], ps->XQ, ps->XS, ps->n_pad, nc, ps->H, ps->ld_h, false, err, m->n_sm, st))
            return 1;
        ta.x = ps->H; ta.ld_x = ps->ld_h; ta.norm_w = nullptr; ta.cols = m->hidden; ta.hidden = m->hidden;
        ta.k_pad = ps->k_pad[PF_K_HID];
        pf_swiglu_quant_kernel<<<nc, 256, (size_t)m->hidden * 4, st>>>(ta);
        CK(cudaGetLastError());
        if (launch_gemm(P.w2, ps->mapB[PF_K_HID], ps->XQ, ps->XS, ps->n_pad, nc, ps->X, m->dim, true, err, m->n_sm, st))
            return 1;
    }
    return 0;
}

int pf_run_layers(EmberCudaState *s, const int *ids_dev, int n, int start) {
    EmberCudaModel *m = s->m;
    if (pf_prepare_model(m) || pf_prepare_state(s)) return 1;
    PfState *ps = s->pf;
    PfSeq q;
    memset(&q, 0, sizeof(q));
    q.kc = s->kc; q.vc = s->vc; q.k_layer = s->k_layer_elems; q.v_layer = s->v_layer_elems;
    q.ctx = s->ctx; q.kstride = s->kstride; q.kv_fp16 = s->kv_fp16; q.rope = s->rope;
    q.p_cap = (int)round_up((size_t)(start + n), 4);
    if (!attn_tile(m, q.p_cap, &q.tq, &q.rs))
        return set_err("prefill: %d positions do not fit the attention tile", start + n);
    int nc = 0;
    for (int c0 = 0; c0 < n; c0 += ps->n_cap) {
        nc = n - c0 < ps->n_cap ? n - c0 : ps->n_cap;
        q.n = nc;
        q.start = start + c0;
        if (pf_layers(m, ps, q, ids_dev + c0, s->ctl + CTL_ERR, s->stream)) return 1;
    }
    // the last token's residual stream feeds the final norm + lm_head
    CK(cudaMemcpyAsync(s->x, ps->X + (size_t)(nc - 1) * m->dim, (size_t)m->dim * 4, cudaMemcpyDeviceToDevice,
                       s->stream));
    return 0;
}

// ------------------------------------------------------------ op level --------

__global__ void __launch_bounds__(256) pf_quant_kernel(const PfTokArgs a) {
    extern __shared__ __align__(16) float pf_row[];
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) pf_row[i] = a.x[(size_t)t * a.ld_x + i];
    __syncthreads();
    pf_quant_row(pf_row, a, t);
}

int pf_matmul_batch(int device, float *out, const float *x, const DevMat &w, int B, void *xq_blocks) {
    if (pf_init(device)) return 1;
    if (w.dtype != EMBER_DT_Q8_0 && w.dtype != EMBER_DT_Q4_0) return set_err("pf_matmul_batch: dtype");
    PfModel pm;
    PfMat pk;
    const DevMat *parts[1] = { &w };
    int rc = build_pack(&pm, &pk, parts, 1);
    const int n_pad = (int)round_up((size_t)B, 128);
    float *dx = nullptr, *dout = nullptr, *dxs = nullptr;
    int8_t *dxq = nullptr;
    int *derr = nullptr;
    CUtensorMap maps[PF_NBN];
    std::vector<void *> tmp;
    if (!rc) rc = pf_alloc(tmp, (void **)&dx, (size_t)B * w.cols * 4) || pf_alloc(tmp, (void **)&dout, (size_t)B * w.rows * 4) ||
                  pf_alloc(tmp, (void **)&dxq, (size_t)n_pad * pk.k_pad) ||
                  pf_alloc(tmp, (void **)&dxs, (size_t)pk.nb * n_pad * 4) || pf_alloc(tmp, (void **)&derr, 16);
    if (!rc && (cudaMemset(dxq, 0, (size_t)n_pad * pk.k_pad) != cudaSuccess || cudaMemset(derr, 0, 16) != cudaSuccess ||
                cudaMemset(dxs, 0, (size_t)pk.nb * n_pad * 4) != cudaSuccess ||
                cudaMemcpy(dx, x, (size_t)B * w.cols * 4, cudaMemcpyHostToDevice) != cudaSuccess))
        rc = set_err("pf_matmul_batch: upload failed");
    for (int j = 0; j < PF_NBN && !rc; j++) rc = map_i8(&maps[j], dxq, (size_t)pk.k_pad, (size_t)n_pad, PF_BNS[j]);
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
    if (!rc) {
        PfTokArgs ta;
        memset(&ta, 0, sizeof(ta));
        ta.x = dx; ta.ld_x = w.cols; ta.cols = w.cols; ta.xq = dxq; ta.k_pad = pk.k_pad; ta.xs = dxs; ta.n_pad = n_pad;
        pf_quant_kernel<<<B, 256, (size_t)w.cols * 4>>>(ta);
        if (cudaGetLastError() != cudaSuccess) rc = set_err("pf_matmul_batch: quant launch failed");
    }
    if (!rc) rc = launch_gemm(pk, maps, dxq, dxs, n_pad, B, dout, w.rows, false, derr, nsm, 0);
    int herr = 0;
    if (!rc && (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost) != cudaSuccess))
        rc = set_err("pf_matmul_batch: %s", cudaGetErrorString(cudaGetLastError()));
    if (!rc && herr) rc = set_err("pf_matmul_batch: device wait timed out (code %d)", herr);
    if (!rc && cudaMemcpy(out, dout, (size_t)B * w.rows * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = set_err("pf_matmul_batch: download failed");
    if (!rc && xq_blocks) {
        // the caller's scratch receives the Q8_0 blocks of every column, as the
        // reference's ember_matmul_batch leaves them (ref src/kernels.c:254-257)
        const int nb = w.cols / 32;
        std::vector<int8_t> hq((size_t)B * pk.k_pad);
        std::vector<float> hs((size_t)nb * n_pad);
        if (cudaMemcpy(hq.data(), dxq, hq.size(), cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(hs.data(), dxs, hs.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = set_err("pf_matmul_batch: download failed");
        BlockQ8_0 *blk = static_cast<BlockQ8_0 *>(xq_blocks);
        for (int b = 0; !rc && b < B; b++)
            for (int j = 0; j < nb; j++) {
                BlockQ8_0 &o = blk[(size_t)b * nb + j];
                o.d = ember_f32_to_f16(hs[(size_t)j * n_pad + b]);   // exact: the value is an fp16
                memcpy(o.qs, hq.data() + (size_t)b * pk.k_pad + (size_t)j * 32, 32);
            }
    }
    for (void *p : tmp) cudaFree(p);
    for (void *p : pm.allocs) cudaFree(p);
    return rc;
}

}  // namespace emb

// ------------------------------------------------------------ streams --------
// Batched greedy decode of independent streams (BASELINE's many-sequence
// workload): every step runs all S streams' tokens through the layers as S
// token rows -- the tensor-core GEMMs read each weight row once per token tile
// -- with each row at its own position in its own KV cache, then the final norm,
// the lm_head GEMM and a per-stream argmax. Per stream the arithmetic is the
// single-token step's, so each stream's tokens equal its own greedy run.

namespace emb {

static int pf_prepare_head(EmberCudaModel *m) {
    if (m->pf->head_ready) return 0;
    if (m->lm_head.dtype == EMBER_DT_F32) return set_err("batched decode needs a quantized lm_head");
    const DevMat *parts[1] = { &m->lm_head };
    if (build_pack(m->pf, &m->pf->head, parts, 1)) return 1;
    CK(cudaDeviceSynchronize());
    m->pf->head_ready = 1;
    return 0;
}

// first index of the strict maximum of each stream's logits (ref
// src/sample.c:114-118); the stream's next token and position; out[step][S]
__global__ void __launch_bounds__(256) batch_argmax_kernel(const float *logits, int ld, int vocab, int *tok,
                                                          int *pos, int *out, const int *nout, int S) {
    __shared__ float sv[256];
    __shared__ int si[256];
    const int s = blockIdx.x, tid = threadIdx.x;
    const float *row = logits + (size_t)s * ld;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = tid; i < vocab; i += 256) {
        const float v = row[i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    sv[tid] = bv;
    si[tid] = bi;
    __syncthreads();
    for (int st = 128; st > 0; st >>= 1) {
        if (tid < st) {
            const float v = sv[tid + st];
            const int i = si[tid + st];
            if (v > sv[tid] || (v == sv[tid] && i < si[tid])) { sv[tid] = v; si[tid] = i; }
        }
        __syncthreads();
    }
    if (tid == 0) {
        // all -inf/NaN, or a NaN at index 0: the reference's loop keeps index 0
        const int idx = (si[0] == 0x7FFFFFFF || isnan(row[0])) ? 0 : si[0];
        tok[s] = idx;
        pos[s] += 1;
        out[(size_t)(*nout) * S + s] = idx;
    }
}

__global__ void batch_advance_kernel(int *nout) {
    if (threadIdx.x == 0) *nout += 1;
}

}  // namespace emb

using namespace emb;

struct EmberCudaBatch {
    EmberCudaModel *m = nullptr;
    int S = 0, ctx = 0, kv_fp16 = 0, max_steps = 0;
    EmberCudaState *worker = nullptr;     // prompt prefill; its cache pointers are aimed at a stream
    void *kc = nullptr, *vc = nullptr;    // [S][layers][...] in the worker's per-layer layout
    size_t stride = 0;                    // elements per stream (keys' and values' caches alike)
    int *tok = nullptr, *pos = nullptr, *out = nullptr, *nout = nullptr;
    float *logits = nullptr;
    int ld_log = 0;
    PfState *ps = nullptr;
    cudaGraphExec_t g_step = nullptr;
    std::vector<void *> allocs;
    // few streams: one single-stream state per stream, their greedy graphs
    // running at once on their own CUDA streams (a handful of one-token steps
    // overlap better than a GEMM of a handful of rows)
    std::vector<EmberCudaState *> reps;
    int *htok = nullptr;                  // pinned [S][max_steps] chosen tokens
};

// streams up to which a batch keeps one single-stream state per stream (the
// default number of hardware work queues); EMBER_BATCH=gemm forces the batched
// GEMM path at any size
constexpr int BATCH_REPLICA_MAX = 8;

static void batch_release(EmberCudaBatch *b) {
    if (b->g_step) cudaGraphExecDestroy(b->g_step);
    pf_state_free(b->ps);
    for (void *p : b->allocs) cudaFree(p);
    b->allocs.clear();
    if (b->worker) ember_cuda_state_free(b->worker);
    for (EmberCudaState *r : b->reps) ember_cuda_state_free(r);
    b->reps.clear();
    if (b->htok) cudaFreeHost(b->htok);
    b->htok = nullptr;
}

extern "C" int ember_cuda_batch_new(EmberCudaModel *m, int n_streams, int ctx, int kv_fp16, const float *rope_cs,
                                    int max_steps, EmberCudaBatch **out) {
    *out = nullptr;
    CK(cudaSetDevice(m->device));
    if (n_streams < 1 || n_streams > PF_CHUNK) return set_err("batch: n_streams must be in [1, %d]", PF_CHUNK);
    if (max_steps < 1) return set_err("batch: max_steps must be positive");
    if (!pf_supported(m)) return set_err("batch: the model's layer weights are not all Q8_0 / Q4_0");
    EmberCudaBatch *b = new EmberCudaBatch();
    b->m = m; b->S = n_streams; b->ctx = ctx; b->kv_fp16 = kv_fp16 ? 1 : 0; b->max_steps = max_steps;
    const char *mode = getenv("EMBER_BATCH");
    if (n_streams <= BATCH_REPLICA_MAX && !(mode && strcmp(mode, "gemm") == 0)) {
        int rc = cudaMallocHost((void **)&b->htok, (size_t)n_streams * max_steps * 4) != cudaSuccess
                     ? set_err("batch: pinned token buffer allocation failed")
                     : 0;
        for (int i = 0; i < n_streams && !rc; i++) {
            EmberCudaState *r = nullptr;
            rc = ember_cuda_state_new(m, ctx, b->kv_fp16, rope_cs, &r);
            if (!rc) b->reps.push_back(r);
            // the replicas run at once on their own streams: the graph step, not the
            // persistent kernel (which takes every SM)
            if (!rc) persist_release(r);
            if (!rc) rc = greedy_prepare(r);
        }
        if (rc) {
            batch_release(b);
            delete b;
            return 1;
        }
        *out = b;
        return 0;
    }
    int rc = ember_cuda_state_new(m, ctx, b->kv_fp16, rope_cs, &b->worker);
    if (!rc) rc = pf_prepare_model(m) || pf_init(m->device) || pf_prepare_head(m);
    const size_t es = b->kv_fp16 ? 2 : 4;
    if (!rc) {
        EmberCudaState *w = b->worker;
        const size_t sk = (size_t)m->n_layers * w->k_layer_elems, sv = (size_t)m->n_layers * w->v_layer_elems;
        b->stride = sk > sv ? sk : sv;
        b->ld_log = m->pf->head.rows_pad;
        rc = pf_alloc(b->allocs, &b->kc, b->stride * es * n_streams + 256) ||
             pf_alloc(b->allocs, &b->vc, b->stride * es * n_streams + 256) ||
             pf_alloc(b->allocs, (void **)&b->tok, (size_t)n_streams * 4) ||
             pf_alloc(b->allocs, (void **)&b->pos, (size_t)n_streams * 4) ||
             pf_alloc(b->allocs, (void **)&b->out, (size_t)max_steps * n_streams * 4) ||
             pf_alloc(b->allocs, (void **)&b->nout, 16) ||
             pf_alloc(b->allocs, (void **)&b->logits, (size_t)n_streams * b->ld_log * 4) ||
             pf_state_new(m, n_streams, &b->ps);
        if (!rc && (cudaMemset(b->kc, 0, b->stride * es * n_streams) != cudaSuccess ||
                    cudaMemset(b->vc, 0, b->stride * es * n_streams) != cudaSuccess))
            rc = set_err("batch: cache initialisation failed");
    }
    if (!rc) {
        // attention of one row per stream: the whole context in the weight tile
        int tq, rs;
        if (!attn_tile(m, (int)round_up((size_t)ctx, 4), &tq, &rs))
            rc = set_err("batch: a context of %d does not fit the attention tile", ctx);
    }
    if (rc) {
        batch_release(b);
        delete b;
        return 1;
    }
    *out = b;
    return 0;
}

extern "C" void ember_cuda_batch_free(EmberCudaBatch *b) {
    if (!b) return;
    cudaSetDevice(b->m->device);
    if (b->worker) cudaStreamSynchronize(b->worker->stream);
    for (EmberCudaState *r : b->reps) cudaStreamSynchronize(r->stream);
    batch_release(b);
    delete b;
}

extern "C" void *ember_cuda_batch_stream(EmberCudaBatch *b) {
    return (void *)(b->worker ? b->worker->stream : b->reps[0]->stream);
}

// the worker state's cache pointers aimed at stream i's cache
static void aim_worker(EmberCudaBatch *b, int i) {
    const size_t es = b->kv_fp16 ? 2 : 4;
    b->worker->kc = (char *)b->kc + (size_t)i * b->stride * es;
    b->worker->vc = (char *)b->vc + (size_t)i * b->stride * es;
}

extern "C" int ember_cuda_batch_prefill(EmberCudaBatch *b, int stream, const int *ids, int n, float *host_logits) {
    CK(cudaSetDevice(b->m->device));
    if (stream < 0 || stream >= b->S) return set_err("batch: stream %d out of range", stream);
    if (n < 1 || n > b->ctx) return set_err("batch: prompt of %d tokens does not fit the context", n);
    if (!b->reps.empty()) return ember_cuda_prefill(b->reps[stream], ids, n, 0, host_logits);
    EmberCudaState *w = b->worker;
    aim_worker(b, stream);
    // the batched prefill (also for one token: the decode graphs of the worker
    // address its own cache, never a stream's)
    return ember_cuda_prefill_batched(w, ids, n, 0, host_logits);
}

// one greedy step of every stream, recorded once into a graph
static int batch_record(EmberCudaBatch *b) {
    EmberCudaModel *m = b->m;
    EmberCudaState *w = b->worker;
    cudaStream_t st = w->stream;
    int *err = w->ctl + CTL_ERR;
    PfSeq q;
    memset(&q, 0, sizeof(q));
    q.n = b->S; q.start = 0; q.pos = b->pos;
    q.kc = b->kc; q.vc = b->vc; q.cache_stride = b->stride;
    q.k_layer = w->k_layer_elems; q.v_layer = w->v_layer_elems;
    q.ctx = b->ctx; q.kstride = w->kstride; q.kv_fp16 = b->kv_fp16; q.rope = w->rope;
    q.p_cap = (int)round_up((size_t)b->ctx, 4);
    q.tq = 1;
    q.rs = (m->n_heads / m->n_kv + 3) / 4 * 4;
    // attention per (kv head, stream) (attn_batch_kernel) where the kv head's query
    // heads fit one CTA, else per (query head, stream) (attn_decode_kernel, BATCH);
    // EMBER_BATCH_ATTN=head forces the latter, =tile the prefill's token-tile
    // kernel (for comparisons)
    const char *ba = getenv("EMBER_BATCH_ATTN");
    q.dec_attn = !(w->att_in_smem && w->m->head_dim <= ATTN_THREADS) || (ba && strcmp(ba, "tile") == 0)
                     ? 0
                     : ((ba && strcmp(ba, "head") == 0) ? 2 : 1);
    // chunks of 48 positions (fp32, head_dim 128: 48 KB of buffers), so several
    // (head, stream) CTAs share an SM; EMBER_BATCH_ATTN_CHUNK overrides (tuning)
    {
        const size_t es = b->kv_fp16 ? 2 : 4, hd = (size_t)m->head_dim;
        const char *ce = getenv("EMBER_BATCH_ATTN_CHUNK");
        int ch = ce && atoi(ce) >= 8 ? atoi(ce) / 8 * 8 : (int)((48 * 1024) / (2 * hd * es)) / 8 * 8;
        if (ch < 8) ch = 8;
        if (ch > w->attn_chunk) ch = w->attn_chunk;
        q.dec_chunk = ch;
        q.dec_smem = 2 * (size_t)ch * hd * es + ((size_t)b->ctx * 4 + 15) / 16 * 16;
    }
    q.ctl = w->ctl;
    if (pf_layers(m, b->ps, q, b->tok, err, st)) return 1;
    // final norm + lm_head over the S rows, then each stream's argmax
    PfState *ps = b->ps;
    PfTokArgs ta;
    memset(&ta, 0, sizeof(ta));
    ta.xq = ps->XQ; ta.xs = ps->XS; ta.n_pad = ps->n_pad; ta.ex = m->ex; ta.eps = m->eps;
    ta.x = ps->X; ta.ld_x = m->dim; ta.norm_w = m->final_norm; ta.cols = m->dim; ta.k_pad = ps->k_pad[PF_K_DIM];
    pf_norm_quant_kernel<<<b->S, 256, (size_t)m->dim * 8, st>>>(ta);
    CK(cudaGetLastError());
    if (launch_gemm(m->pf->head, ps->mapB[PF_K_DIM], ps->XQ, ps->XS, ps->n_pad, b->S, b->logits, b->ld_log, false, err,
                    m->n_sm, st))
        return 1;
    batch_argmax_kernel<<<b->S, 256, 0, st>>>(b->logits, b->ld_log, m->vocab, b->tok, b->pos, b->out, b->nout, b->S);
    CK(cudaGetLastError());
    batch_advance_kernel<<<1, 32, 0, st>>>(b->nout);
    CK(cudaGetLastError());
    return 0;
}

extern "C" int ember_cuda_batch_greedy(EmberCudaBatch *b, const int *toks, const int *pos, int n_steps,
                                       int *host_tokens, float *host_logits) {
    CK(cudaSetDevice(b->m->device));
    if (n_steps < 1 || n_steps > b->max_steps) return set_err("batch: n_steps must be in [1, %d]", b->max_steps);
    for (int i = 0; i < b->S; i++) {
        if (toks[i] < 0 || toks[i] >= b->m->vocab) return set_err("batch: token id %d out of range", toks[i]);
        if (pos[i] < 0 || pos[i] + n_steps > b->ctx) return set_err("batch: stream %d does not fit the context", i);
    }
    if (!b->reps.empty()) {
        // every stream's steps enqueued before any wait, so that they run at once
        for (int i = 0; i < b->S; i++)
            if (greedy_enqueue(b->reps[i], toks[i], pos[i], n_steps, b->htok + (size_t)i * b->max_steps)) {
                // streams 0..i-1 still copy their tokens into the pinned buffer:
                // wait for them before reporting the failure
                for (int j = 0; j < i; j++) cudaStreamSynchronize(b->reps[j]->stream);
                return 1;
            }
        int rc = 0;
        for (int i = 0; i < b->S; i++) rc |= greedy_finish(b->reps[i]);
        if (rc) return 1;
        if (host_tokens)
            for (int t = 0; t < n_steps; t++)
                for (int i = 0; i < b->S; i++) host_tokens[(size_t)t * b->S + i] = b->htok[(size_t)i * b->max_steps + t];
        if (host_logits)
            for (int i = 0; i < b->S; i++)
                CK(cudaMemcpy(host_logits + (size_t)i * b->m->vocab, b->reps[i]->logits, (size_t)b->m->vocab * 4,
                              cudaMemcpyDeviceToHost));
        return 0;
    }
    cudaStream_t st = b->worker->stream;
    if (!b->g_step) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = batch_record(b);
        cudaError_t e = cudaStreamEndCapture(st, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return 1;
        }
        if (e != cudaSuccess) return set_err("batch graph capture failed: %s", cudaGetErrorString(e));
        e = cudaGraphInstantiate(&b->g_step, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return set_err("batch graph instantiate failed: %s", cudaGetErrorString(e));
    }
    CK(cudaMemcpyAsync(b->tok, toks, (size_t)b->S * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(b->pos, pos, (size_t)b->S * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemsetAsync(b->nout, 0, 4, st));
    CK(cudaMemsetAsync(b->worker->ctl + CTL_ERR, 0, 4, st));
    for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(b->g_step, st));
    if (host_tokens)
        CK(cudaMemcpyAsync(host_tokens, b->out, (size_t)n_steps * b->S * 4, cudaMemcpyDeviceToHost, st));
    if (host_logits)
        CK(cudaMemcpy2DAsync(host_logits, (size_t)b->m->vocab * 4, b->logits, (size_t)b->ld_log * 4,
                             (size_t)b->m->vocab * 4, (size_t)b->S, cudaMemcpyDeviceToHost, st));
    int herr = 0;
    CK(cudaMemcpyAsync(&herr, b->worker->ctl + CTL_ERR, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (herr) return set_err("batch: device wait timed out (code %d)", herr);
    return 0;
}

#ifdef EMBER_PROBES
// profiling build only: the last GEMM launch's trace (1024 timestamps)
extern "C" int ember_cuda_pf_trace_read(unsigned long long *out, unsigned long long *cta) {
    if (cudaDeviceSynchronize() != cudaSuccess) return 1;
    if (cta && cudaMemcpyFromSymbol(cta, emb::g_pf_cta, sizeof(emb::g_pf_cta)) != cudaSuccess) return 1;
    return cudaMemcpyFromSymbol(out, emb::g_pf_trace, sizeof(emb::g_pf_trace)) != cudaSuccess;
}
#endif
