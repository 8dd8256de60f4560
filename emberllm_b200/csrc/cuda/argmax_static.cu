// argmax_static.cu — greedy token selection over logits already on the GPU,
// without any device allocation.
//
// Who needs this. Some programs that embed this library cannot let it allocate
// device memory: a serving host that hands the whole GPU to its own memory pool
// up front and treats any outside cudaMalloc as an error, code that must not
// pay the device-wide synchronisation cudaMalloc/cudaFree can imply on a
// per-token path, or a caller whose device memory budget is fixed in advance.
// The library's other greedy path keeps its argmax scratch in the run state,
// which ember_state_new allocates; this entry point instead works on buffers the
// caller already owns: it reads `n` device floats and writes one device int.
//
// Scratch. The per-block partial maxima and the completion ticket live in the
// file-scope array below, of fixed size (kMaxBlocks blocks, about 2 KB). Every
// GPU that loads the library holds one copy until the process exits. All calls
// on a device share it and it keeps the last call's contents, so the ticket is
// cleared at the start of every call; two calls whose work overlaps on the GPU
// (e.g. issued on different streams without ordering) race on it and may return
// wrong indices.
//
// Set-up. The first call on each device (the device that owns `logits`) looks up
// the array's device address with cudaGetSymbolAddress while that device is
// current, and caches it. Make that first call before any stream capture is
// begun on the calling thread. The call selects that device to enqueue its work
// and selects the caller's current device again before it returns.
#include <cuda_runtime.h>

#include <pthread.h>
#include <stdio.h>

#include "ember_cuda.h"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 256;
constexpr int kMaxDevices = 64;
constexpr long long kMaxN = 1LL << 26;   // 67,108,864 logits per call

// [0, kMaxBlocks) float partial maxima, then kMaxBlocks int indices, then the ticket
constexpr size_t kScratchBytes = (size_t)kMaxBlocks * 8 + 256;
static __device__ __align__(256) unsigned char g_argmax_scratch[kScratchBytes];

void *g_scratch_addr[kMaxDevices];
pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;

__device__ __forceinline__ void take(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// first index of the strict maximum of x[0..n) (the reference's greedy pick,
// src/sample.c:114-118: best = 0, then i wins when x[i] > x[best]). So a NaN
// never wins, an all -inf/NaN input gives 0, and a NaN at index 0 gives 0 (no
// value compares greater than it)
__global__ void __launch_bounds__(kThreads) argmax_static_kernel(const float *x, int n, int *out,
                                                                 unsigned char *scratch) {
    float *part_v = reinterpret_cast<float *>(scratch);
    int *part_i = reinterpret_cast<int *>(scratch + (size_t)kMaxBlocks * 4);
    unsigned *ticket = reinterpret_cast<unsigned *>(scratch + (size_t)kMaxBlocks * 8);
    __shared__ float sv[kThreads];
    __shared__ int si[kThreads];
    __shared__ bool last;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < n; i += (long long)gridDim.x * kThreads)
        take(bv, bi, x[i], (int)i);
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int st = kThreads / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            float v = sv[threadIdx.x];
            int i = si[threadIdx.x];
            take(v, i, sv[threadIdx.x + st], si[threadIdx.x + st]);
            sv[threadIdx.x] = v;
            si[threadIdx.x] = i;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        part_v[blockIdx.x] = sv[0];
        part_i[blockIdx.x] = si[0];
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // the last block to finish merges every block's partial
    bv = -INFINITY;
    bi = 0x7FFFFFFF;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads)
        take(bv, bi, *(volatile float *)&part_v[b], *(volatile int *)&part_i[b]);
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int st = kThreads / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            float v = sv[threadIdx.x];
            int i = si[threadIdx.x];
            take(v, i, sv[threadIdx.x + st], si[threadIdx.x + st]);
            sv[threadIdx.x] = v;
            si[threadIdx.x] = i;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *out = (si[0] == 0x7FFFFFFF || isnan(x[0])) ? 0 : si[0];
        *ticket = 0u;
    }
}

// status codes of ember_cuda_argmax_static (a line on stderr explains each)
enum { kOk = 0, kBadSize = 1, kBadPointer = 2, kCudaError = 3 };

int report(int code, const char *what, const char *detail) {
    fprintf(stderr, "ember: ember_cuda_argmax_static: %s%s%s\n", what, detail ? ": " : "", detail ? detail : "");
    return code;
}

// the device that owns device memory p, or -1 when p is not device memory
int device_of(const void *p) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return attr.type == cudaMemoryTypeDevice ? attr.device : -1;
}

int argmax_static_on(int dev, const float *logits, int n, int *out_index, cudaStream_t st) {
    cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) return report(kCudaError, "cannot select the logits' device", cudaGetErrorString(e));
#if CUDART_VERSION >= 12080
    if (st) {
        int sdev = -1;
        if (cudaStreamGetDevice(st, &sdev) != cudaSuccess) {
            cudaGetLastError();
            return report(kBadPointer, "stream is not a valid CUDA stream", nullptr);
        }
        if (sdev != dev) return report(kBadPointer, "stream belongs to another device than logits", nullptr);
    }
#endif
    // once per device, with that device current: the scratch array's device address
    pthread_mutex_lock(&g_mu);
    if (!g_scratch_addr[dev]) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_argmax_scratch);
        if (e != cudaSuccess) {
            pthread_mutex_unlock(&g_mu);
            return report(kCudaError, "cudaGetSymbolAddress failed", cudaGetErrorString(e));
        }
        g_scratch_addr[dev] = ptr;
    }
    unsigned char *scratch = (unsigned char *)g_scratch_addr[dev];
    pthread_mutex_unlock(&g_mu);
    const long long want = ((long long)n + kThreads * 4 - 1) / (kThreads * 4);
    const int grid = (int)(want < kMaxBlocks ? want : kMaxBlocks);
    // the completion ticket must start at zero: the array keeps the last call's contents
    e = cudaMemsetAsync(scratch + (size_t)kMaxBlocks * 8, 0, sizeof(unsigned), st);
    if (e == cudaSuccess) {
        argmax_static_kernel<<<grid, kThreads, 0, st>>>(logits, n, out_index, scratch);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return report(kCudaError, "launch failed", cudaGetErrorString(e));
    return kOk;
}

}  // namespace

extern "C" int ember_cuda_argmax_static(const float *logits, int n, int *out_index, void *stream) {
    if (n < 1 || (long long)n > kMaxN) {
        char d[96];
        snprintf(d, sizeof(d), "n = %d, allowed 1..%lld", n, kMaxN);
        return report(kBadSize, "size outside the supported range", d);
    }
    if (!logits || !out_index) return report(kBadPointer, "null logits or output pointer", nullptr);
    const int dev = device_of(logits);
    if (dev < 0) return report(kBadPointer, "logits is not device memory", nullptr);
    if (dev >= kMaxDevices) return report(kBadPointer, "device index too large", nullptr);
    if (device_of(out_index) != dev) return report(kBadPointer, "out_index is not device memory of the logits' device", nullptr);
    // the kernel runs on the logits' device; the caller's current device is put back
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) {
        cudaGetLastError();
        prev = -1;
    }
    const int rc = argmax_static_on(dev, logits, n, out_index, (cudaStream_t)stream);
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    return rc;
}
