/*
 * utils.h -- the reference's math helpers (src/utils.h) on host tensors, computed on the GPU.
 *
 * These exist so that code written against the reference's utilities keeps working; each call copies
 * its host operands to the current CUDA device, runs the library's kernel and copies the result
 * back.  The decode path (transformer.h: forward) does not go through them.
 */
#ifndef DIOLKOS_UTILS_H
#define DIOLKOS_UTILS_H

#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct Tensor Tensor;

bool reliable_isnan(double x);
size_t round_down_32(size_t i);

/* softmax over the first `size` values, in place (src/utils.c:39-57). */
void softmax(Tensor *x, int size);
void softmax_f32(float *x, int size);
/* o = rmsnorm(x) * weight over `size` values (src/utils.c:59-76); F32 tensors. */
void rmsnorm(Tensor *o, Tensor *x, Tensor *weight, int size);
/* xout[d] = W[d x n] * x[n] for a Q8_0 W and F32 x / xout (matmul_Q8_0, src/utils.c:106-138):
 * bit-identical to the reference build.  W is packed for the GPU on its first use and the packed copy
 * is kept (keyed by the tensor) until the process exits. */
void matmul(Tensor *xout, Tensor *x, Tensor *w, int n, int d);

/* Kept for source compatibility: the library needs no scratch set-up. */
void init_utils(int dim, int hidden_dim);

#ifdef __cplusplus
}
#endif
#endif
