/* threads.c — emberllm's thread-pool API kept as no-ops.
 *
 * emberllm splits matmul rows and attention heads over a pthread pool
 * (ref src/threads.c:61-104). Here the CUDA grid does that work, but the CLI
 * (`--threads N`, ref src/main.c:179) and the server (ref src/server.c:477) still
 * call these functions, so they stay callable: init records the count,
 * parallel_for runs the range inline on the calling thread. */
#include "ember_ops.h"

static int g_requested_threads = 1;

void ember_threads_init(int nthreads) { g_requested_threads = nthreads < 1 ? 1 : nthreads; }

void ember_threads_shutdown(void) { g_requested_threads = 1; }

int ember_nthreads(void) { return g_requested_threads; }

void ember_parallel_for(EmberRangeFn fn, void *ctx, int n) {
    if (n > 0) fn(ctx, 0, n);
}

int ember_should_parallel(long work) {
    (void)work;
    return 0;
}
