/*
 * ref_driver.c -- a thin C driver over the UNMODIFIED reference sources (test infrastructure).
 *
 * It is compiled together with the reference's own src/{tensor,utils,transformer,safetensors,
 * parson,sampler,tokenizer}.c (read in place, never copied) by oracle/Makefile, with the
 * reference's own flags, into oracle/_ref/<variant>/liboracle_ref.so.  Tests and the CPU
 * baseline call it through ctypes.  Every entry point below only marshals plain buffers into the
 * reference's Tensor structs and calls the reference function named beside it.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <omp.h>

#include "safetensors.h"
#include "sampler.h"
#include "tensor.h"
#include "transformer.h"
#include "utils.h"

typedef struct ORef {
    Transformer t;
    Sampler greedy;
} ORef;

static int g_utils_dim = 0;

/* matmul_Q8_0 (utils.c:106) quantises into the global scratch that init_utils (utils.c:102)
 * allocates; make sure it is large enough for `n` inputs. */
static void ensure_utils(int n) {
    if (n > g_utils_dim) {
        init_utils(n, n);
        g_utils_dim = n;
    }
}

/* build_transformer_from_safetensors (transformer.c:32).  The reference keeps its Q8_0 cache at
 * cache/<basename(model_dir)>/ relative to the working directory and creates only the last
 * directory level (safetensors.c:103-104), so the driver enters `work_dir`, creates `cache/`,
 * loads, and returns to the caller's working directory. */
void *oref_load(const char *model_dir, const char *work_dir) {
    char old[PATH_MAX];
    if (!getcwd(old, sizeof old)) return NULL;
    if (chdir(work_dir) != 0) return NULL;
    mkdir("cache", 0755);
    ORef *h = calloc(1, sizeof(ORef));
    build_transformer_from_safetensors(&h->t, model_dir);
    if (chdir(old) != 0) { /* the model is loaded; the old cwd vanished */ }
    build_sampler(&h->greedy, h->t.config.vocab_size, 0.0f, 0.9f, 1);
    if (h->t.config.dim > g_utils_dim) g_utils_dim = h->t.config.dim;
    if (h->t.config.hidden_dim > g_utils_dim) g_utils_dim = h->t.config.hidden_dim;
    return h;
}

void oref_config(void *hp, int *out7) {
    ORef *h = hp;
    const Config *c = &h->t.config;
    out7[0] = c->dim; out7[1] = c->hidden_dim; out7[2] = c->n_layers; out7[3] = c->n_heads;
    out7[4] = c->n_kv_heads; out7[5] = c->vocab_size; out7[6] = c->seq_len;
}

/* forward (transformer.c:55); copies the returned logits (RunState.logits, F32[vocab]). */
void oref_forward(void *hp, int token, int pos, float *logits) {
    ORef *h = hp;
    Tensor *lg = forward(&h->t, token, pos);
    memcpy(logits, lg->data, sizeof(float) * (size_t)h->t.config.vocab_size);
}

/* Copy of the residual stream x after the last forward (RunState.x, which forward() overwrites
 * with rmsnorm(x) at transformer.c:234). */
void oref_state_x(void *hp, float *out) {
    ORef *h = hp;
    memcpy(out, h->t.state.x->data, sizeof(float) * (size_t)h->t.config.dim);
}

/* The bf16 KV-cache rows of positions [pos0, pos0 + n) of one layer (RunState key_cache /
 * value_cache, [layer][pos][kv_dim], transformer.c:25-26, written at :145-146). */
void oref_kv_rows(void *hp, int layer, int pos0, int n, uint16_t *k, uint16_t *v) {
    ORef *h = hp;
    const Config *c = &h->t.config;
    const size_t kv_dim = (size_t)c->dim * c->n_kv_heads / c->n_heads;
    const size_t off = ((size_t)layer * c->seq_len + pos0) * kv_dim;
    memcpy(k, (uint16_t *)h->t.state.key_cache->data + off, sizeof(uint16_t) * kv_dim * (size_t)n);
    memcpy(v, (uint16_t *)h->t.state.value_cache->data + off, sizeof(uint16_t) * kv_dim * (size_t)n);
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* The OpenMP thread count the reference's parallel loops use: n > 0 sets it (omp_set_num_threads,
 * overriding OMP_NUM_THREADS, which a multi-process launcher may have set to 1); returns the count
 * in effect. */
int oref_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}

/* The greedy token loop of generate (localinfer.c:42-99) fed with token ids instead of a text
 * prompt: prompt tokens are forced one position at a time, the next token is sampled with the
 * reference's sample() at temperature 0 once the prompt is consumed, the loop stops when the
 * sampled token is 1, and the clock starts after the first forward.  Returns the number of
 * generated (non-forced) tokens written to out; *tok_s gets the reference's tok/s figure.
 * Optional (NULL: skipped): *gen_s = wall seconds of the positions that produced the generated
 * tokens (forward + sample, from position n_prompt-1 on); top2[2*i], top2[2*i+1] = the two largest
 * logits at the position that produced generated token i. */
int oref_generate(void *hp, const int *prompt, int n_prompt, int steps, int *out, double *tok_s, double *gen_s,
                  float *top2) {
    ORef *h = hp;
    const int vocab = h->t.config.vocab_size;
    int token = prompt[0], pos = 0, n_out = 0;
    double start = 0.0, gen0 = 0.0;
    while (pos < steps) {
        if (pos == n_prompt - 1) gen0 = now_s();
        Tensor *lg = forward(&h->t, token, pos);
        int next;
        if (pos < n_prompt - 1) {
            next = prompt[pos + 1];
        } else {
            if (top2) {
                const float *l = (const float *)lg->data;
                float a = -INFINITY, b = -INFINITY;
                for (int i = 0; i < vocab; i++) {
                    if (l[i] > a) { b = a; a = l[i]; }
                    else if (l[i] > b) b = l[i];
                }
                top2[2 * n_out] = a;
                top2[2 * n_out + 1] = b;
            }
            next = sample(&h->greedy, (float *)lg->data);
            out[n_out++] = next;
        }
        pos++;
        if (next == 1) break;
        token = next;
        if (start == 0.0) start = now_s();
    }
    const double end = now_s();
    if (tok_s) *tok_s = (pos > 1) ? (double)(pos - 1) / (end - start) : 0.0;
    if (gen_s) *gen_s = (n_out > 0) ? end - gen0 : 0.0;
    return n_out;
}

/* convert_f32_q8_slice_into_offset (tensor.c:199): activation quantisation. */
void oref_quant_f32(const float *x, size_t n, int8_t *q, float *s) {
    Tensor *in = tensor_create(n, F32);
    Tensor *dst = tensor_create(n, Q8_0);
    memcpy(in->data, x, n * sizeof(float));
    convert_f32_q8_slice_into_offset(dst, in, 0, n, 0);
    memcpy(q, dst->data, n);
    memcpy(s, dst->scale, n / 32 * sizeof(float));
    tensor_destroy(in);
    tensor_destroy(dst);
}

/* convert (tensor.c:374) from BF16 to Q8_0, i.e. convert_bf16_q8_0 (tensor.c:312): the load-time
 * weight quantiser. */
void oref_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s) {
    Tensor *in = tensor_create(n, BF16);
    memcpy(in->data, x, n * sizeof(uint16_t));
    Tensor *dst = convert(in, Q8_0);
    memcpy(q, dst->data, n);
    memcpy(s, dst->scale, n / 32 * sizeof(float));
    tensor_destroy(in);
    tensor_destroy(dst);
}

/* A prepared Q8_0 matrix for repeated matmul calls (utils.c:185 -> matmul_Q8_0 utils.c:106). */
typedef struct OMat { Tensor *w, *x, *out; int n, d; } OMat;

void *oref_mat_create(const int8_t *wq, const float *ws, int n, int d) {
    OMat *m = calloc(1, sizeof(OMat));
    size_t nd = (size_t)n * (size_t)d;
    m->w = tensor_create(nd, Q8_0);
    memcpy(m->w->data, wq, nd);
    memcpy(m->w->scale, ws, nd / 32 * sizeof(float));
    m->x = tensor_create((size_t)n, F32);
    m->out = tensor_create((size_t)d, F32);
    m->n = n; m->d = d;
    ensure_utils(n);
    return m;
}

void oref_mat_run(void *mp, const float *x, float *out) {
    OMat *m = mp;
    memcpy(m->x->data, x, (size_t)m->n * sizeof(float));
    matmul(m->out, m->x, m->w, m->n, m->d);
    memcpy(out, m->out->data, (size_t)m->d * sizeof(float));
}

/* Time `iters` back-to-back matmul calls on the prepared matrix (the loop of benchmark.c:42-46,
 * on an arbitrary [d x n] shape).  Returns seconds. */
double oref_mat_time(void *mp, int iters) {
    OMat *m = mp;
    double t0 = now_s();
    for (int i = 0; i < iters; i++) matmul(m->out, m->x, m->w, m->n, m->d);
    return now_s() - t0;
}

void oref_mat_destroy(void *mp) {
    OMat *m = mp;
    tensor_destroy(m->w);
    tensor_destroy(m->x);
    tensor_destroy(m->out);
    free(m);
}

/* rmsnorm (utils.c:59). */
void oref_rmsnorm(float *o, const float *x, const float *w, int n) {
    Tensor *to = tensor_create((size_t)n, F32), *tx = tensor_create((size_t)n, F32),
           *tw = tensor_create((size_t)n, F32);
    memcpy(tx->data, x, (size_t)n * 4);
    memcpy(tw->data, w, (size_t)n * 4);
    rmsnorm(to, tx, tw, n);
    memcpy(o, to->data, (size_t)n * 4);
    tensor_destroy(to); tensor_destroy(tx); tensor_destroy(tw);
}

/* softmax_f32 (utils.c:39), in place. */
void oref_softmax(float *x, int n) { softmax_f32(x, n); }

/* sample (sampler.c:108) with temperature 0 -> sample_argmax (sampler.c:6). */
int oref_argmax(const float *logits, int n) {
    Sampler s;
    build_sampler(&s, n, 0.0f, 0.9f, 1);
    float *copy = malloc((size_t)n * sizeof(float));
    memcpy(copy, logits, (size_t)n * sizeof(float));
    int r = sample(&s, copy);
    free(copy);
    free_sampler(&s);
    return r;
}

/* sample (sampler.c:108) with temperature/top-p and the reference's xorshift state; the logits are
 * mutated in place like the reference does.  Returns the token and advances *rng. */
int oref_sample(float *logits, int n, float temperature, float topp, unsigned long long *rng) {
    Sampler s;
    build_sampler(&s, n, temperature, topp, *rng);
    int r = sample(&s, logits);
    *rng = s.rng_state;
    free_sampler(&s);
    return r;
}
