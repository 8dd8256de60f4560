// wait_check.cu — TEST HOOK, built into libember_testhooks.so only: makes the
// product's bounded device waits run out (a barrier nothing completes, a
// hand-off word nothing writes) with a short limit, so a test can check that
// the wait returns, records its error code and leaves the context usable.
#include "cuda/persist.cuh"
#include "ember_testhooks.h"

namespace emb {

__global__ void __launch_bounds__(PTT) wait_timeout_kernel(int mode, unsigned tries, int *ctl,
                                                          const unsigned long long *word, int *ok) {
    __shared__ __align__(8) uint64_t bar;
    const int tid = threadIdx.x;
    if (mode == 0) {
        if (tid == 0) {
            mbar_init(&bar, 1);   // one arrival expected; none comes
            fence_mbar_init();
        }
        __syncthreads();
        if (tid == 0) *ok = mbar_wait_n(&bar, 0, ctl + CTL_ERR, ERR_GEMV_WAIT, tries) ? 1 : 0;
    } else if (tid < PT) {
        PArgs a;
        memset(&a, 0, sizeof(a));
        a.ctl = ctl;
        a.spin_limit = tries;
        uint32_t v = 0;
        const bool r = tw_wait1(&v, word, 7u, a);   // tag 7: never written
        if (tid == 0) *ok = r ? 1 : 0;
    }
}

}  // namespace emb

using namespace emb;

extern "C" int ember_testhook_wait_timeout(int mode, unsigned tries, int *ok_out, int *err_out, float *ms_out) {
    int *ctl = nullptr, *ok = nullptr;
    unsigned long long *word = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 1;
    if (cudaMalloc(&ctl, CTL_WORDS * 4) == cudaSuccess && cudaMalloc(&ok, 4) == cudaSuccess &&
        cudaMalloc(&word, 8) == cudaSuccess && cudaMemset(ctl, 0, CTL_WORDS * 4) == cudaSuccess &&
        cudaMemset(ok, 0xff, 4) == cudaSuccess && cudaMemset(word, 0, 8) == cudaSuccess &&
        cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess) {
        cudaEventRecord(e0);
        wait_timeout_kernel<<<1, PTT>>>(mode, tries, ctl, word, ok);
        cudaEventRecord(e1);
        if (cudaGetLastError() == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
            cudaMemcpy(ok_out, ok, 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
            cudaMemcpy(err_out, ctl + CTL_ERR, 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
            cudaEventElapsedTime(ms_out, e0, e1) == cudaSuccess)
            rc = 0;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(ctl);
    cudaFree(ok);
    cudaFree(word);
    return rc;
}
