/* model_internal.h — host-side definitions shared by io.c and model.c. */
#ifndef EMBER_B200_MODEL_INTERNAL_H
#define EMBER_B200_MODEL_INTERNAL_H

#include "ember.h"
#include "ember_cuda.h"
#include "ember_ops.h"

#include <stddef.h>
#include <stdint.h>

/* the mmap'd file (as in ref src/io.c:18-24) plus its device weights */
struct EmberModel {
    int fd;
    size_t size;
    const uint8_t *base;
    const EmberHeader *hdr;
    const EmberTensor *table;
    EmberCudaModel *dev;   /* uploaded by the first ember_state_new_ex; NULL before */
};

#endif /* EMBER_B200_MODEL_INTERNAL_H */
