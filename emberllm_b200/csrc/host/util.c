/* util.c — fatal errors and checked allocation, keeping emberllm's convention
 * (ref src/util.c:8-34): a fatal error prints "ember: <message>" to stderr and
 * exits with status 1; allocators never hand back NULL. */
#include "ember_ops.h"

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

void ember_die(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "ember: ");
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
    fflush(stderr);
    exit(1);
}

void *ember_xmalloc(size_t n, const char *what) {
    void *p = malloc(n > 0 ? n : 1);
    if (p == NULL) ember_die("out of memory allocating %s (%zu bytes)", what, n);
    return p;
}

void *ember_xcalloc(size_t count, size_t size, const char *what) {
    void *p = calloc(count > 0 ? count : 1, size > 0 ? size : 1);
    if (p == NULL) ember_die("out of memory allocating %s (%zu x %zu bytes)", what, count, size);
    return p;
}

void *ember_xrealloc(void *p, size_t n, const char *what) {
    void *q = realloc(p, n > 0 ? n : 1);
    if (q == NULL) ember_die("out of memory reallocating %s (%zu bytes)", what, n);
    return q;
}
