/*
 * ref_hooks.c -- per-layer checkpoints of the reference's forward() (test infrastructure).
 *
 * oracle/Makefile compiles the reference's UNMODIFIED src/transformer.c a second time with
 *     -Drmsnorm=oref_hook_rmsnorm -Dmatmul=oref_hook_matmul
 * so that forward() (transformer.c:55-239) calls the two functions below instead of rmsnorm
 * (utils.c:59) and matmul (utils.c:185).  Each hook records its input and then calls the real
 * function, so the arithmetic of forward() is unchanged (tests/test_oracle.py checks that the
 * hooked build's logits equal the plain build's bit for bit).  This file is compiled without the
 * renaming, with the reference's own flags, and linked into _ref/<variant>/liboracle_ref_hooked.so.
 *
 * What one forward() records (L layers, calls in forward()'s order):
 *   rmsnorm inputs   x before layer l's attention rmsnorm (transformer.c:76), x after its
 *                    attention residual (:204), ... and the final x (:234): 2L+1 vectors of dim --
 *                    the residual stream after every residual add, the embedding row first;
 *   matmul inputs    per layer the calls wq, wk, wv (:83-85), wo (:196), w1, w3 (:208-209),
 *                    w2 (:225), then wcls (:237).  Only the four distinct activations per layer
 *                    are kept -- wq's (rmsnorm(x)), wo's (attention output), w1's (rmsnorm(x)),
 *                    w2's (SwiGLU output) -- and wcls's: the fp32 input vector and the Q8_0 form
 *                    matmul_Q8_0 (utils.c:106-107) quantised it to (int8 values, fp32 group scales),
 *                    read back from the reference's own scratch tensor temp_q8 (utils.c:101).
 */
#include <stdint.h>
#include <string.h>

#include "tensor.h"
#include "transformer.h"
#include "utils.h"

extern Tensor *temp_q8;  /* utils.c:101: the activation scratch matmul_Q8_0 quantises into */

typedef struct HookRec {
    int on;
    int dim, hidden, n_layers;
    int n_rms, n_mm;        /* calls seen in this forward */
    float *xres;            /* [2L+1][dim] */
    float *ain;             /* the kept matmul inputs, concatenated */
    int8_t *aq;
    float *as;
    size_t aoff;            /* elements written to ain / aq so far */
} HookRec;

static HookRec g_rec;

void oref_hook_begin(int dim, int hidden, int n_layers, float *xres, float *ain, int8_t *aq, float *as) {
    g_rec.on = 1;
    g_rec.dim = dim;
    g_rec.hidden = hidden;
    g_rec.n_layers = n_layers;
    g_rec.n_rms = 0;
    g_rec.n_mm = 0;
    g_rec.xres = xres;
    g_rec.ain = ain;
    g_rec.aq = aq;
    g_rec.as = as;
    g_rec.aoff = 0;
}

/* Number of rmsnorm and matmul calls the last recorded forward made (2L+1 and 7L+1 expected). */
void oref_hook_end(int *n_rms, int *n_mm) {
    g_rec.on = 0;
    *n_rms = g_rec.n_rms;
    *n_mm = g_rec.n_mm;
}

void oref_hook_rmsnorm(Tensor *o, Tensor *x, Tensor *weight, int size) {
    if (g_rec.on && g_rec.n_rms < 2 * g_rec.n_layers + 1 && size == g_rec.dim)
        memcpy(g_rec.xres + (size_t)g_rec.n_rms * size, x->data, sizeof(float) * (size_t)size);
    if (g_rec.on) g_rec.n_rms++;
    rmsnorm(o, x, weight, size);
}

void oref_hook_matmul(Tensor *xout, Tensor *x, Tensor *w, int n, int d) {
    int keep = 0;
    if (g_rec.on) {
        const int c = g_rec.n_mm, k = c % 7;
        keep = (c < 7 * g_rec.n_layers) ? (k == 0 || k == 3 || k == 4 || k == 6) : (c == 7 * g_rec.n_layers);
        if (keep) memcpy(g_rec.ain + g_rec.aoff, x->data, sizeof(float) * (size_t)n);
        g_rec.n_mm++;
    }
    matmul(xout, x, w, n, d);
    if (keep) {
        memcpy(g_rec.aq + g_rec.aoff, temp_q8->data, (size_t)n);
        memcpy(g_rec.as + g_rec.aoff / 32, temp_q8->scale, sizeof(float) * (size_t)(n / 32));
        g_rec.aoff += (size_t)n;
    }
}

/* forward() (transformer.c:55) with the checkpoints above recorded.  hp is a handle from oref_load
 * (ref_driver.c), whose first member is the reference's Transformer.  counts[0..1] receive the
 * numbers of rmsnorm and matmul calls (2L+1 and 7L+1). */
void oref_forward_dump(void *hp, int token, int pos, float *logits, float *xres, float *ain, int8_t *aq, float *as,
                       int *counts) {
    Transformer *t = (Transformer *)hp;
    const Config *c = &t->config;
    oref_hook_begin(c->dim, c->hidden_dim, c->n_layers, xres, ain, aq, as);
    Tensor *lg = forward(t, token, pos);
    oref_hook_end(&counts[0], &counts[1]);
    memcpy(logits, lg->data, sizeof(float) * (size_t)c->vocab_size);
}
