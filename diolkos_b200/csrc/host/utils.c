/*
 * utils.c -- the reference's math helpers (src/utils.c) on host tensors, computed on the current
 * CUDA device with the library's kernels.
 *
 * matmul keeps the packed GPU copy of each weight matrix it has seen (keyed by the tensor, its data
 * pointer and the shape), so repeated calls on the same weights stream only the activation and the
 * result over PCIe; tensor_destroy drops the copy.  Not re-entrant, like the reference (which
 * shares one scratch tensor, src/utils.c:101).
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "diolkos.h"
#include "host_internal.h"
#include "tensor.h"
#include "utils.h"

bool reliable_isnan(double x) {
    uint64_t bits;
    memcpy(&bits, &x, sizeof bits);
    return ((bits >> 52) & 0x7FF) == 0x7FF && (bits & ((1ull << 52) - 1)) != 0;
}

size_t round_down_32(size_t i) { return i & ~(size_t)31; }

void init_utils(int dim, int hidden_dim) {
    (void)dim;
    (void)hidden_dim;
}

static dev_buf g_a, g_b, g_c;

void softmax_f32(float *x, int size) {
    if (size <= 0) return;
    float *d = dev_reserve(&g_a, (size_t)size * sizeof(float));
    host_check_cuda(cudaMemcpy(d, x, (size_t)size * sizeof(float), cudaMemcpyHostToDevice), "softmax: copy in");
    host_check(dk_softmax(d, size, NULL), "softmax");
    host_check_cuda(cudaMemcpy(x, d, (size_t)size * sizeof(float), cudaMemcpyDeviceToHost), "softmax: copy out");
}

void softmax(Tensor *x, int size) { softmax_f32(data_f32(x), size); }

void rmsnorm(Tensor *o, Tensor *x, Tensor *weight, int size) {
    if (size <= 0) return;
    const size_t bytes = (size_t)size * sizeof(float);
    float *dx = dev_reserve(&g_a, bytes), *dw = dev_reserve(&g_b, bytes);
    host_check_cuda(cudaMemcpy(dx, data_f32(x), bytes, cudaMemcpyHostToDevice), "rmsnorm: copy x");
    host_check_cuda(cudaMemcpy(dw, data_f32(weight), bytes, cudaMemcpyHostToDevice), "rmsnorm: copy weight");
    host_check(dk_rmsnorm(dx, dx, dw, size, NULL), "rmsnorm");
    host_check_cuda(cudaMemcpy(data_f32(o), dx, bytes, cudaMemcpyDeviceToHost), "rmsnorm: copy out");
}

/* ---- packed weights seen by matmul ----------------------------------------------------------- */
typedef struct packed_w {
    const Tensor *t;
    const void *data;
    int n, d, device;
    uint8_t *packed;
    struct packed_w *next;
} packed_w;

static packed_w *g_packed;

static const uint8_t *packed_weight(Tensor *w, int n, int d) {
    int dev = 0;
    host_check_cuda(cudaGetDevice(&dev), "matmul: cudaGetDevice");
    for (packed_w *e = g_packed; e; e = e->next)
        if (e->t == w && e->data == (const void *)w->data && e->n == n && e->d == d && e->device == dev)
            return e->packed;
    const size_t vals = (size_t)n * (size_t)d;
    const size_t bytes = dk_q8_packed_bytes(n, d);
    if (!bytes) {
        fprintf(stderr, "diolkos: matmul: unsupported shape n=%d d=%d\n", n, d);
        exit(EXIT_FAILURE);
    }
    int8_t *q = dev_reserve(&g_b, vals);
    float *s = dev_reserve(&g_c, vals / 32 * sizeof(float));
    host_check_cuda(cudaMemcpy(q, data_i8(w), vals, cudaMemcpyHostToDevice), "matmul: copy weight values");
    host_check_cuda(cudaMemcpy(s, w->scale, vals / 32 * sizeof(float), cudaMemcpyHostToDevice),
                    "matmul: copy weight scales");
    packed_w *e = host_calloc(1, sizeof(packed_w));
    host_check_cuda(cudaMalloc((void **)&e->packed, bytes), "matmul: cudaMalloc (packed weight)");
    host_check(dk_q8_pack(e->packed, n, d, q, s, NULL), "matmul: pack weight");
    e->t = w;
    e->data = w->data;
    e->n = n;
    e->d = d;
    e->device = dev;
    e->next = g_packed;
    g_packed = e;
    return e->packed;
}

void utils_forget_tensor(const Tensor *t) {
    for (packed_w **pp = &g_packed; *pp;) {
        packed_w *e = *pp;
        if (e->t == t) {
            *pp = e->next;
            int cur = 0;
            cudaGetDevice(&cur);
            cudaSetDevice(e->device);
            cudaFree(e->packed);
            cudaSetDevice(cur);
            free(e);
        } else {
            pp = &e->next;
        }
    }
}

void matmul(Tensor *xout, Tensor *x, Tensor *w, int n, int d) {
    if (w->type != Q8_0) {
        fprintf(stderr, "diolkos: matmul: %s weights are not supported (this build runs Q8_0 matrices)\n",
                quant_t_to_string(w->type));
        exit(EXIT_FAILURE);
    }
    if (n <= 0 || d <= 0 || n % 32 || w->dim < (size_t)n * (size_t)d || x->dim < (size_t)n || xout->dim < (size_t)d) {
        fprintf(stderr, "diolkos: matmul: bad shape n=%d d=%d (w %zu, x %zu, out %zu elements)\n", n, d, w->dim,
                x->dim, xout->dim);
        exit(EXIT_FAILURE);
    }
    const uint8_t *pw = packed_weight(w, n, d);
    float *dx = dev_reserve(&g_a, ((size_t)n + (size_t)d) * sizeof(float));
    float *dout = dx + ((n + 3) & ~3);
    host_check_cuda(cudaMemcpy(dx, data_f32(x), (size_t)n * sizeof(float), cudaMemcpyHostToDevice), "matmul: copy x");
    host_check(dk_matmul_q8_0(dout, dx, pw, n, d, NULL), "matmul");
    host_check_cuda(cudaMemcpy(data_f32(xout), dout, (size_t)d * sizeof(float), cudaMemcpyDeviceToHost),
                    "matmul: copy out");
}
