/* io.c — .ember loading (replaces ref src/io.c:30-96).
 *
 * The file is mmap'd read-only and validated with the reference's checks, in
 * its order and with its messages, so malformed-file behaviour (NULL + a line on
 * stderr, never a crash) is unchanged. The model additionally owns the device
 * copy of its weights, which the first state created for it uploads
 * (csrc/host/model.c) and ember_model_free releases.
 */
#include "model_internal.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static EmberModel *load_fail(const char *why, void *map, size_t len, int fd) {
    fprintf(stderr, "ember: %s\n", why);
    if (map) munmap(map, len);
    if (fd >= 0) close(fd);
    return NULL;
}

EmberModel *ember_model_load(const char *path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return load_fail("cannot open model file", NULL, 0, -1);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < (off_t)sizeof(EmberHeader))
        return load_fail("model file too small", NULL, 0, fd);
    size_t len = (size_t)st.st_size;
    void *map = mmap(NULL, len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) return load_fail("mmap failed", NULL, 0, fd);

    const EmberHeader *h = (const EmberHeader *)map;
    uint64_t fsize = (uint64_t)len;
    if (memcmp(h->magic, "EMBR", 4) != 0 || h->version != EMBER_VERSION)
        return load_fail("bad magic or version", map, len, fd);
    if (h->n_tensors < 0 || h->dim <= 0 || h->n_layers <= 0 || h->vocab_size <= 0)
        return load_fail("header has non-positive dimensions", map, len, fd);
    if (h->tensor_table_offset > fsize ||
        h->tensor_table_size > fsize - h->tensor_table_offset ||
        h->tensor_table_size < (uint64_t)h->n_tensors * sizeof(EmberTensor))
        return load_fail("tensor table out of bounds", map, len, fd);
    if (h->tokenizer_offset > fsize || h->tokenizer_size > fsize - h->tokenizer_offset)
        return load_fail("tokenizer blob out of bounds", map, len, fd);

    EmberModel *m = ember_xcalloc(1, sizeof(*m), "EmberModel");
    m->fd = fd;
    m->size = len;
    m->base = (const uint8_t *)map;
    m->hdr = h;
    m->table = (const EmberTensor *)(m->base + h->tensor_table_offset);
    m->dev = NULL;
    madvise(map, len, MADV_WILLNEED);
    return m;
}

void ember_model_free(EmberModel *m) {
    if (!m) return;
    if (m->dev) ember_cuda_model_free(m->dev);
    munmap((void *)m->base, m->size);
    close(m->fd);
    free(m);
}

const EmberHeader *ember_model_header(const EmberModel *m) { return m->hdr; }

const EmberTensor *ember_model_tensor(const EmberModel *m, const char *name) {
    for (int i = 0; i < m->hdr->n_tensors; i++)
        if (strncmp(m->table[i].name, name, sizeof(m->table[i].name)) == 0) return &m->table[i];
    return NULL;
}

const void *ember_model_data(const EmberModel *m, const EmberTensor *t) {
    if (!t) return NULL;
    if (t->offset + t->nbytes > m->size) {
        fprintf(stderr, "ember: tensor data out of bounds\n");
        return NULL;
    }
    return m->base + t->offset;
}
