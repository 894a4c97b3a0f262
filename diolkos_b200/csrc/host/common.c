/*
 * common.c -- exit-on-error helpers and device staging buffers for the reference-API host library.
 * The reference's entry points return no errors: they print to stderr and exit(EXIT_FAILURE)
 * (src/safetensors.c:21-23, :362-399; asserts elsewhere); these keep that behaviour on top of the
 * library's status codes.
 */
#include <stdio.h>
#include <stdlib.h>

#include <cuda_runtime_api.h>

#include "diolkos.h"
#include "host_internal.h"

void host_check(int status, const char *what) {
    if (status == DK_OK) return;
    fprintf(stderr, "diolkos: %s: %s\n", what, dk_last_error());
    exit(EXIT_FAILURE);
}

void host_check_cuda(int e, const char *what) {
    if (e == 0) return;
    fprintf(stderr, "diolkos: %s: %s\n", what, cudaGetErrorString((cudaError_t)e));
    exit(EXIT_FAILURE);
}

void *host_malloc(size_t n) {
    void *p = malloc(n ? n : 1);
    if (!p) {
        fprintf(stderr, "diolkos: out of host memory (%zu bytes)\n", n);
        exit(EXIT_FAILURE);
    }
    return p;
}

void *host_calloc(size_t n, size_t size) {
    void *p = calloc(n ? n : 1, size ? size : 1);
    if (!p) {
        fprintf(stderr, "diolkos: out of host memory (%zu x %zu bytes)\n", n, size);
        exit(EXIT_FAILURE);
    }
    return p;
}

void *dev_reserve(dev_buf *b, size_t bytes) {
    int dev = 0;
    host_check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (b->ptr && b->device == dev && bytes <= b->bytes) return b->ptr;
    if (b->ptr) {
        if (b->device != dev) host_check_cuda(cudaSetDevice(b->device), "cudaSetDevice");
        host_check_cuda(cudaFree(b->ptr), "cudaFree");
        if (b->device != dev) host_check_cuda(cudaSetDevice(dev), "cudaSetDevice");
    }
    b->ptr = NULL;
    b->bytes = 0;
    host_check_cuda(cudaMalloc(&b->ptr, bytes ? bytes : 16), "cudaMalloc (staging buffer)");
    b->bytes = bytes;
    b->device = dev;
    return b->ptr;
}
