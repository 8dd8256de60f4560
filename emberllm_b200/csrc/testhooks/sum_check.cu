// sum_check.cu — TEST HOOK, built into libember_testhooks.so only (never into
// the product library): runs split_chain_sum (the RMSNorm sum of squares of the
// decode GEMVs, csrc/cuda/common.cuh) on a batch of vectors, one 256-thread block
// per vector, reporting the sum and whether the split evaluation answered or the
// rest was added sequentially.
#include "cuda/persist.cuh"
#include "ember_testhooks.h"

namespace emb {

__global__ void __launch_bounds__(256) split_sum_check_kernel(const float *v, int n, float *out, int *hit) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *t = reinterpret_cast<float *>(smem);
    const float *x = v + (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += 256) t[i] = x[i];
    __syncthreads();
    int h = 0;
    const float s = split_chain_sum<256>(t, n, &h);
    if (threadIdx.x == 0) {
        out[blockIdx.x] = s;
        hit[blockIdx.x] = h;
    }
}

// the persistent step's 512-thread variant (psum, csrc/cuda/persist.cuh)
__global__ void __launch_bounds__(PT) psum_check_kernel(const float *v, int n, float *out) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *t = reinterpret_cast<float *>(smem);
    const float *x = v + (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += PT) t[i] = x[i];
    __syncthreads();
    const float s = psum(t, n);
    if (threadIdx.x == 0) out[blockIdx.x] = s;
}

}  // namespace emb

using namespace emb;

extern "C" int ember_cuda_psum_batch(const float *host_terms, int n, int count, float *host_out) {
    if (n < 16 || n % 16 || count < 1 || n > 32768) return 1;
    const size_t smem = (size_t)n * 4, vb = (size_t)n * count * sizeof(float);
    float *dv = nullptr, *dout = nullptr;
    int rc = 1;
    if (cudaMalloc(&dv, vb) != cudaSuccess || cudaMalloc(&dout, (size_t)count * 4) != cudaSuccess) goto done;
    if (cudaMemcpy(dv, host_terms, vb, cudaMemcpyHostToDevice) != cudaSuccess) goto done;
    if (cudaFuncSetAttribute(psum_check_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        goto done;
    psum_check_kernel<<<count, PT, smem>>>(dv, n, dout);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) goto done;
    if (cudaMemcpy(host_out, dout, (size_t)count * 4, cudaMemcpyDeviceToHost) != cudaSuccess) goto done;
    rc = 0;
done:
    cudaFree(dv);
    cudaFree(dout);
    return rc;
}

extern "C" int ember_cuda_split_sum_batch(const float *host_terms, int n, int count, float *host_out, int *host_hit) {
    if (n < 1 || count < 1 || n > 32768) return 1;
    const size_t smem = (size_t)n * 4;
    float *dv = nullptr, *dout = nullptr;
    int *dhit = nullptr;
    const size_t vb = (size_t)n * count * sizeof(float);
    int rc = 1;
    if (cudaMalloc(&dv, vb) != cudaSuccess || cudaMalloc(&dout, (size_t)count * 4) != cudaSuccess ||
        cudaMalloc(&dhit, (size_t)count * 4) != cudaSuccess)
        goto done;
    if (cudaMemcpy(dv, host_terms, vb, cudaMemcpyHostToDevice) != cudaSuccess) goto done;
    if (cudaFuncSetAttribute(split_sum_check_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        goto done;
    split_sum_check_kernel<<<count, 256, smem>>>(dv, n, dout, dhit);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) goto done;
    if (cudaMemcpy(host_out, dout, (size_t)count * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(host_hit, dhit, (size_t)count * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        goto done;
    rc = 0;
done:
    cudaFree(dv);
    cudaFree(dout);
    cudaFree(dhit);
    return rc;
}
