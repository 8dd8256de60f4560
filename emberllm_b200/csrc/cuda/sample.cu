// sample.cu — the reference's sampler (src/sample.c:76-175) on the device, over
// the logits of a state's last step, so a token can be drawn without copying
// the vocabulary's logits to the host and sorting them there.
//
// The steps and their arithmetic are the reference's, in its order:
//   penalties  over the history in array order, one thread (ref :76-96)
//   greedy     temperature <= 0: the first index of the maximum (ref :114-127)
//   logits / temperature, max = logits[argmax], e = expf(l - max) (the host C
//              library's expf, reproduced by expf_exact), sum = sequential fp32
//              sum in index order, p = e / sum (ref :129-135)
//   candidates (p, index) in descending p; the reference sorts with qsort,
//              which on this platform's C library is stable (measured), so ties
//              keep index order: here a bitonic sort of the total order (p
//              descending, index ascending) gives the same sequence
//   truncation top_k, min_p (against the largest p), top_p (cumulative sum in
//              sorted order), cutoff, then r = u * cutoff and the first
//              candidate whose running sum exceeds r (ref :137-172)
// u is the reference's xorshift64* draw, computed on the host (the caller's
// rng state advances exactly as in the reference). Sequential fp32 sums run on
// one thread while the rest of its CTA stages the next chunk into shared memory.
#include <cuda_runtime.h>

#include <string.h>

#include "common.cuh"
#include "runtime_internal.cuh"

using namespace emb;

namespace emb {

constexpr int SM_THREADS = 256;
constexpr int SM_CHUNK = 4096;          // elements staged per chunk (two buffers)
constexpr int SM_TILE = 2048;           // bitonic tile sorted in shared memory

struct SampleBufs {
    float *w = nullptr;                 // working logits / exponentials [vocab]
    unsigned long long *keys = nullptr; // [npow2] sort keys
    int *hist = nullptr;                // [hist_cap] history copy
    int hist_cap = 0;
    float *part_v = nullptr;            // argmax partials
    int *part_i = nullptr;
    float *res_f = nullptr;             // [0] max, [1] sum
    int *res_i = nullptr;               // [0] argmax, [1] chosen
    int npow2 = 0, nblk = 0;
};

struct SampleArgs {
    float temperature, top_p, min_p, repeat_penalty, presence_penalty, frequency_penalty, u;
    int top_k, hist_len, n;
};

__global__ void smp_copy(const float *logits, float *w, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) w[i] = logits[i];
}

// repetition / presence / frequency penalties (ref src/sample.c:76-96): the
// history in array order; repetition and presence at a token's first entry,
// frequency at every entry
__global__ void smp_penalties(float *w, const int *hist, SampleArgs a) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const bool has_rep = a.repeat_penalty != 1.0f, has_freq = a.frequency_penalty != 0.0f,
               has_pres = a.presence_penalty != 0.0f;
    if (!has_rep && !has_freq && !has_pres) return;
    for (int i = 0; i < a.hist_len; i++) {
        const int t = hist[i];
        if (t < 0 || t >= a.n) continue;
        bool first = true;
        for (int j = 0; j < i; j++)
            if (hist[j] == t) { first = false; break; }
        if (first) {
            if (has_rep) w[t] = w[t] > 0.0f ? fdiv(w[t], a.repeat_penalty) : fmul(w[t], a.repeat_penalty);
            if (has_pres) w[t] = fsub(w[t], a.presence_penalty);
        }
        if (has_freq) w[t] = fsub(w[t], a.frequency_penalty);
    }
}

__global__ void smp_div(float *w, int n, float temperature) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) w[i] = fdiv(w[i], temperature);
}

EMB_DEV void am_take(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// first index of the strict maximum, per block, then merged in block order
__global__ void __launch_bounds__(SM_THREADS) smp_argmax_part(const float *w, int n, float *pv, int *pi) {
    __shared__ float sv[SM_THREADS];
    __shared__ int si[SM_THREADS];
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = blockIdx.x * SM_THREADS + threadIdx.x; i < n; i += gridDim.x * SM_THREADS) am_take(bv, bi, w[i], i);
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int st = SM_THREADS / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            float v = sv[threadIdx.x];
            int i = si[threadIdx.x];
            am_take(v, i, sv[threadIdx.x + st], si[threadIdx.x + st]);
            sv[threadIdx.x] = v;
            si[threadIdx.x] = i;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) { pv[blockIdx.x] = sv[0]; pi[blockIdx.x] = si[0]; }
}

// the merge; a NaN at index 0 keeps index 0 (ref src/sample.c:114-118: nothing
// compares greater than it); res_f[0] = the maximum's value
__global__ void smp_argmax_final(const float *w, const float *pv, const int *pi, int nblk, float *res_f, int *res_i) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int b = 0; b < nblk; b++) am_take(bv, bi, pv[b], pi[b]);
    const int idx = (bi == 0x7FFFFFFF || isnan(w[0])) ? 0 : bi;
    res_i[0] = idx;
    res_i[1] = idx;
    res_f[0] = w[idx];
}

// e = expf(l - max), in place
__global__ void smp_exp(float *w, int n, const float *res_f, ExpfDev ex) {
    __shared__ double tab[64];
    expf_table_load(tab, ex);
    __syncthreads();
    const float mx = res_f[0];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        w[i] = expf_exact(ex, tab, fsub(w[i], mx));
}

// Stage chunk c of src (SM_CHUNK elements) into buf by threads first..255.
template <typename T>
EMB_DEV void stage_chunk(T *buf, const T *src, int c, int n, int first) {
    const int base = c * SM_CHUNK;
    for (int i = threadIdx.x - first; i < SM_CHUNK && base + i < n; i += SM_THREADS - first) buf[i] = src[base + i];
}

// sum = ((0 + e[0]) + e[1]) + ... in index order (ref src/sample.c:133): thread 0
// adds one staged chunk while the other threads stage the next
__global__ void __launch_bounds__(SM_THREADS) smp_sum(const float *w, int n, float *res_f) {
    __shared__ __align__(16) float buf[2][SM_CHUNK];
    const int nch = (n + SM_CHUNK - 1) / SM_CHUNK;
    float s = 0.0f;
    stage_chunk(buf[0], w, 0, n, 0);
    __syncthreads();
    for (int c = 0; c < nch; c++) {
        if (threadIdx.x == 0) s = chain_sum(s, buf[c & 1], min(SM_CHUNK, n - c * SM_CHUNK));
        else if (c + 1 < nch) stage_chunk(buf[(c + 1) & 1], w, c + 1, n, 1);   // thread 0 is busy: the others stage
        __syncthreads();
    }
    if (threadIdx.x == 0) res_f[1] = s;
}

// p = e / sum and its sort key: the float bits inverted (p >= 0, so bits order
// as values) above the index, so ascending keys are descending p, then
// ascending index; keys past n sort last
__global__ void smp_keys(const float *w, int n, int npow2, const float *res_f, unsigned long long *keys) {
    const float sum = res_f[1];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npow2; i += gridDim.x * blockDim.x) {
        if (i < n) {
            const float p = fdiv(w[i], sum);
            keys[i] = ((unsigned long long)(~__float_as_uint(p)) << 32) | (unsigned)i;
        } else {
            keys[i] = ~0ull;
        }
    }
}

// ---- bitonic sort of keys[0..npow2), ascending ----
EMB_DEV void cswap(unsigned long long &x, unsigned long long &y, bool asc) {
    if ((x > y) == asc) { const unsigned long long t = x; x = y; y = t; }
}

// every stage k <= SM_TILE inside one tile (k_lo = 2), or, for a stage k > SM_TILE,
// its passes j < SM_TILE (k_lo = k)
__global__ void __launch_bounds__(SM_TILE / 2) smp_bitonic_tile(unsigned long long *keys, int k_lo, int k_hi) {
    __shared__ unsigned long long t[SM_TILE];
    const int base = blockIdx.x * SM_TILE, tid = threadIdx.x;
    t[tid] = keys[base + tid];
    t[tid + SM_TILE / 2] = keys[base + tid + SM_TILE / 2];
    __syncthreads();
    for (int k = k_lo; k <= k_hi; k <<= 1) {
        for (int j = (k_lo == k_hi && k > SM_TILE ? SM_TILE / 2 : k / 2); j > 0; j >>= 1) {
            const int i = 2 * j * (tid / j) + (tid % j), l = i + j;
            const bool asc = ((base + i) & k) == 0;
            cswap(t[i], t[l], asc);
            __syncthreads();
        }
    }
    keys[base + tid] = t[tid];
    keys[base + tid + SM_TILE / 2] = t[tid + SM_TILE / 2];
}

// one pass (k, j) with j >= SM_TILE over the whole array: one pair per thread
__global__ void smp_bitonic_pass(unsigned long long *keys, int npow2, int k, int j) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= npow2 / 2) return;
    const int i = 2 * j * (p / j) + (p % j), l = i + j;
    unsigned long long x = keys[i], y = keys[l];
    const bool asc = (i & k) == 0;
    if ((x > y) == asc) { keys[i] = y; keys[l] = x; }
}

EMB_DEV float key_p(unsigned long long k) { return __uint_as_float(~(uint32_t)(k >> 32)); }
EMB_DEV int key_i(unsigned long long k) { return (int)(uint32_t)(k & 0xFFFFFFFFu); }

// The running sum over cand[0..cnt) continued from *sum, 16 candidates at a time:
// the loads go out first, the additions form a clean dependent chain (entries
// past cnt add +0, which leaves a non-negative sum unchanged), and the running
// sums are tested afterwards. Returns the first index whose running sum meets
// the test (top-p: sum >= lim; draw: lim < sum), with *sum the running sum
// there, or -1 with *sum the sum of all cnt terms -- the reference's loops'
// additions and stopping point exactly.
template <bool DRAW>
EMB_DEV int pick_walk(const unsigned long long *cand, int cnt, float lim, float *sum) {
    float s = *sum;
    for (int i0 = 0; i0 < cnt; i0 += 16) {
        float pv[16], rs[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const float v = key_p(cand[i0 + j]);   // within the staged chunk
            pv[j] = i0 + j < cnt ? v : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            s = fadd(s, pv[j]);
            rs[j] = s;
        }
        int hit = -1;
#pragma unroll
        for (int j = 15; j >= 0; j--)
            if (i0 + j < cnt && (DRAW ? lim < rs[j] : rs[j] >= lim)) hit = j;
        if (hit >= 0) {
            *sum = rs[hit];
            return i0 + hit;
        }
    }
    *sum = s;
    return -1;
}

// The truncation and the draw over the sorted candidates (ref src/sample.c:
// 139-172), thread 0 walking staged chunks of the sorted keys in order.
__global__ void __launch_bounds__(SM_THREADS) smp_pick(const unsigned long long *keys, SampleArgs a, int *res_i) {
    __shared__ unsigned long long buf[2][SM_CHUNK / 2];
    __shared__ int s_m, s_done;
    __shared__ float s_cutoff;
    constexpr int CH = SM_CHUNK / 2;
    const int n = a.n;
    int m = n;
    if (a.top_k > 0 && a.top_k < m) m = a.top_k;
    // min-p: the prefix with p >= min_p * p_max, 16 keys loaded ahead of the tests
    if (threadIdx.x == 0) {
        if (a.min_p > 0.0f && a.min_p < 1.0f) {
            const float thresh = fmul(a.min_p, key_p(keys[0]));
            int keep = 1;
            for (;;) {
                float pv[16];
#pragma unroll
                for (int j = 0; j < 16; j++) pv[j] = keep + j < m ? key_p(keys[keep + j]) : -1.0f;
                int pass = 16;
#pragma unroll
                for (int j = 15; j >= 0; j--)
                    if (!(pv[j] >= thresh)) pass = j;   // the first candidate below the threshold
                keep += pass;
                if (pass < 16 || keep >= m) break;
            }
            m = keep < m ? keep : m;
        }
        s_m = m;
        s_done = 0;
    }
    __syncthreads();
    m = s_m;
    const int nch = (m + CH - 1) / CH;
    // pass 1: top-p over the sorted prefix, or the cutoff as the prefix's sum
    float cum = 0.0f;
    int last = m - 1;
    const bool top_p = a.top_p > 0.0f && a.top_p < 1.0f;
    for (int c = 0; c < nch; c++) {
        const int base = c * CH, cnt = min(CH, m - base);
        for (int i = threadIdx.x; i < cnt; i += SM_THREADS) buf[0][i] = keys[base + i];
        __syncthreads();
        if (threadIdx.x == 0 && !s_done) {
            const int hit = pick_walk<false>(buf[0], cnt, top_p ? a.top_p : INFINITY, &cum);
            if (hit >= 0) {
                last = base + hit;
                s_done = 1;
            }
        }
        __syncthreads();
        if (s_done) break;
    }
    if (threadIdx.x == 0) {
        if (top_p) m = last + 1;
        s_m = m;
        s_cutoff = cum;
        s_done = 0;
    }
    __syncthreads();
    m = s_m;
    // pass 2: r = u * cutoff, the first candidate whose running sum exceeds r
    const float r = fmul(a.u, s_cutoff);
    float run = 0.0f;
    int chosen = 0;
    if (threadIdx.x == 0) chosen = key_i(keys[m - 1]);
    const int nch2 = (m + CH - 1) / CH;
    for (int c = 0; c < nch2; c++) {
        const int base = c * CH, cnt = min(CH, m - base);
        for (int i = threadIdx.x; i < cnt; i += SM_THREADS) buf[1][i] = keys[base + i];
        __syncthreads();
        if (threadIdx.x == 0 && !s_done) {
            const int hit = pick_walk<true>(buf[1], cnt, r, &run);
            if (hit >= 0) {
                chosen = key_i(buf[1][hit]);
                s_done = 1;
            }
        }
        __syncthreads();
        if (s_done) break;
    }
    if (threadIdx.x == 0) res_i[1] = chosen;
}

int sample_bufs(EmberCudaState *s, int hist_len) {
    EmberCudaModel *m = s->m;
    SampleBufs *b = s->sb;
    if (!b) {
        b = new SampleBufs();
        int np = SM_TILE;
        while (np < m->vocab) np <<= 1;
        b->npow2 = np;
        b->nblk = m->n_sm;
        if (salloc(s, (void **)&b->w, (size_t)m->vocab * 4) || salloc(s, (void **)&b->keys, (size_t)np * 8) ||
            salloc(s, (void **)&b->part_v, (size_t)b->nblk * 4) || salloc(s, (void **)&b->part_i, (size_t)b->nblk * 4) ||
            salloc(s, (void **)&b->res_f, 16) || salloc(s, (void **)&b->res_i, 16)) {
            delete b;
            return 1;
        }
        s->sb = b;
    }
    if (hist_len > b->hist_cap) {
        int cap = 64;
        while (cap < hist_len) cap <<= 1;
        if (salloc(s, (void **)&b->hist, (size_t)cap * 4)) return 1;
        b->hist_cap = cap;
    }
    return 0;
}

void sample_release(EmberCudaState *s) {
    delete s->sb;
    s->sb = nullptr;
}

}  // namespace emb

extern "C" int ember_cuda_sample(EmberCudaState *s, const EmberSampleParams *p, float u, const int *hist,
                                 int hist_len, int *out_token) {
    CK(cudaSetDevice(s->m->device));
    if (hist_len < 0 || (hist_len > 0 && !hist)) return set_err("sample: bad history");
    if (!p || !out_token) return set_err("sample: null settings or output");
    if (p->temperature != p->temperature) return set_err("sample: temperature is NaN");
    if (sample_bufs(s, hist_len)) return 1;
    SampleBufs *b = s->sb;
    const int n = s->m->vocab;
    cudaStream_t st = s->stream;
    SampleArgs a;
    a.temperature = p->temperature; a.top_p = p->top_p; a.min_p = p->min_p;
    a.repeat_penalty = p->repeat_penalty; a.presence_penalty = p->presence_penalty;
    a.frequency_penalty = p->frequency_penalty; a.u = u; a.top_k = p->top_k; a.hist_len = hist_len; a.n = n;
    const int grid = s->m->n_sm * 2;
    smp_copy<<<grid, 256, 0, st>>>(s->logits, b->w, n);
    if (hist_len > 0) {
        CK(cudaMemcpyAsync(b->hist, hist, (size_t)hist_len * 4, cudaMemcpyHostToDevice, st));
        smp_penalties<<<1, 32, 0, st>>>(b->w, b->hist, a);
    }
    const bool greedy = p->temperature <= 0.0f;
    if (!greedy) smp_div<<<grid, 256, 0, st>>>(b->w, n, p->temperature);
    smp_argmax_part<<<b->nblk, SM_THREADS, 0, st>>>(b->w, n, b->part_v, b->part_i);
    smp_argmax_final<<<1, 32, 0, st>>>(b->w, b->part_v, b->part_i, b->nblk, b->res_f, b->res_i);
    if (!greedy) {
        smp_exp<<<grid, 256, 0, st>>>(b->w, n, b->res_f, s->m->ex);
        smp_sum<<<1, SM_THREADS, 0, st>>>(b->w, n, b->res_f);
        smp_keys<<<grid, 256, 0, st>>>(b->w, n, b->npow2, b->res_f, b->keys);
        const int ntile = b->npow2 / SM_TILE;
        smp_bitonic_tile<<<ntile, SM_TILE / 2, 0, st>>>(b->keys, 2, SM_TILE);
        for (int k = 2 * SM_TILE; k <= b->npow2; k <<= 1) {
            for (int j = k / 2; j >= SM_TILE; j >>= 1)
                smp_bitonic_pass<<<(b->npow2 / 2 + 255) / 256, 256, 0, st>>>(b->keys, b->npow2, k, j);
            smp_bitonic_tile<<<ntile, SM_TILE / 2, 0, st>>>(b->keys, k, k);
        }
        smp_pick<<<1, SM_THREADS, 0, st>>>(b->keys, a, b->res_i);
    }
    CK(cudaGetLastError());
    int res[2] = {0, 0};
    CK(cudaMemcpyAsync(res, b->res_i, sizeof(res), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    *out_token = res[1];
    return 0;
}
