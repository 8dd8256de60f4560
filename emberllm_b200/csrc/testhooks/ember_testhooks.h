/* ember_testhooks.h — entry points of libember_testhooks.so, a TEST-ONLY library
 * built beside the product (emberllm_b200/libember_testhooks.so). They run
 * device helpers of the product's kernels in isolation for the tests; nothing in
 * the product links or calls them, and they are not part of the C-ABI boundary.
 * Each returns 0 on success. */
#ifndef EMBER_TESTHOOKS_H
#define EMBER_TESTHOOKS_H

#ifdef __cplusplus
extern "C" {
#endif

/* The decode GEMVs' RMSNorm sum (split_chain_sum) on `count` vectors of n
 * non-negative terms each (host arrays, n <= 32768): host_out[i] = the terms
 * added in index order from 0, host_hit[i] = 1 where the split evaluation
 * answered (0: the rest was added sequentially). */
int ember_cuda_split_sum_batch(const float *host_terms, int n, int count, float *host_out, int *host_hit);

/* The persistent token step's 512-thread sum (psum: up to 16 segments) on
 * `count` vectors of n non-negative terms (n a multiple of 16, <= 32768). */
int ember_cuda_psum_batch(const float *host_terms, int n, int count, float *host_out);

/* Copy `bytes` from host memory to a device pointer that the product library
 * allocated (e.g. a state's logits), on the device that owns it: tests plant
 * inputs for a kernel that reads state buffers. */
int ember_testhook_copy_to_device(void *dev_dst, const void *host_src, unsigned long long bytes);

/* A wait that runs out, on the device: mode 0 the mbarrier wait of the kernels'
 * copies (mbar_wait_n) on a barrier nothing completes, mode 1 the persistent
 * step's tagged hand-off wait (tw_wait1) on a word nothing writes; `tries`
 * bounds it (try_wait slices / polls). *ok_out = 1 if the wait reported
 * success, *err_out = the error word afterwards, *ms_out the kernel's time.
 * Returns 0 when the launch itself completed. */
int ember_testhook_wait_timeout(int mode, unsigned tries, int *ok_out, int *err_out, float *ms_out);

#ifdef __cplusplus
}
#endif

#endif
