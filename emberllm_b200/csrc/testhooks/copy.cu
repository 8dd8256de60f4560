// copy.cu — test-only host-to-device copy into product-owned buffers.
#include <cuda_runtime.h>

#include "ember_testhooks.h"

extern "C" int ember_testhook_copy_to_device(void *dev_dst, const void *host_src, unsigned long long bytes) {
    if (!dev_dst || !host_src) return 1;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, dev_dst) != cudaSuccess || at.type != cudaMemoryTypeDevice) return 1;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(at.device) != cudaSuccess) return 1;
    const cudaError_t e = cudaMemcpy(dev_dst, host_src, (size_t)bytes, cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    return e == cudaSuccess ? 0 : 1;
}
