/*
 * port.c -- CPU restatement of the reference's per-token decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the oracle).  Nothing in the product loads or links this file; only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may.  The restatement is
 * pinned against the reference itself (oracle/_ref, compiled from the unmodified reference
 * sources with the reference's -Ofast flags) by tests/test_oracle.py, and against the committed
 * fixtures in tests/golden/.
 *
 * Compiled with -ffp-contract=off -fno-fast-math: every floating-point operation below is the
 * one written, in the order written.  Where the reference's -Ofast build evaluates an expression
 * differently from its source text, the restatement writes out what the compiled reference does
 * and says so.
 */
#include "port.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_bits_to_f32(uint16_t b) {
    union { uint32_t u; float f; } v = { (uint32_t)b << 16 };
    return v.f;
}

/* Upper 16 bits of the fp32 pattern: bf16 by truncation (src/tensor.c:162-178). */
static inline uint16_t f32_to_bf16_trunc(float f) {
    union { float f; uint32_t u; } v = { f };
    return (uint16_t)(v.u >> 16);
}

/* The quantised value of one element: (int8_t)nearbyintf(x * inv), round-half-even.  A
 * non-finite product (an all-zero group has scale 0, inv = +inf and 0*inf = NaN; a denormal scale
 * overflows inv to inf) is undefined behaviour in the reference's cast; on x86 the conversion
 * returns INT_MIN, whose low byte is 0, and this restatement (like the CUDA path) defines it as 0. */
static inline int8_t q8_round(float x, float inv) {
    float v = x * inv;
    if (!(fabsf(v) <= 128.0f)) return 0;
    return (int8_t)(int)nearbyintf(v);
}

/* Q8_0 group quantiser shared by both entry points below.
 *
 * src/tensor.c:327-339 (bf16 weights) computes max_val = max|x|, max_val /= 127,
 * inv = 1.0f / max_val, q = nearbyintf(x * inv).  src/tensor.c:213-226 (fp32 activations) writes
 * max_val /= 127 and nearbyintf(x / max_val); the reference is built with -Ofast, which turns the
 * division by the constant 127 into a multiply by the rounded reciprocal (1.0f/127.0f) and the
 * per-element division into a multiply by the hoisted reciprocal 1.0f/max_val.  Both paths
 * therefore compute exactly:
 *     scale = amax * (1.0f/127.0f);  inv = 1.0f / scale;  q = rint(x * inv).
 * tests/test_oracle.py checks this bit for bit against the compiled reference. */
static void quant_group(const float *x, int8_t *q, float *s) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    const float scale = amax * (1.0f / 127.0f);
    const float inv = 1.0f / scale;
    *s = scale;
    for (int j = 0; j < 32; j++) q[j] = q8_round(x[j], inv);
}

void port_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s) {
    #pragma omp parallel for schedule(static)
    for (size_t g = 0; g < n / 32; g++) {
        float f[32];
        for (int j = 0; j < 32; j++) f[j] = bf16_bits_to_f32(x[g * 32 + j]);
        quant_group(f, q + g * 32, s + g);
    }
}

void port_quant_f32(const float *x, size_t n, int8_t *q, float *s) {
    for (size_t g = 0; g < n / 32; g++) quant_group(x + g * 32, q + g * 32, s + g);
}

/* src/tensor.c:258-263: out = (float)q * scale. */
void port_dequant(const int8_t *q, const float *s, size_t n, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = (float)q[i] * s[i / 32];
}

/* src/utils.c:122-127: exact int32 dot of one 32-element group. */
static inline int32_t group_dot(const int8_t *a, const int8_t *b) {
    int32_t acc = 0;
    for (int k = 0; k < 32; k++) acc += (int32_t)a[k] * (int32_t)b[k];
    return acc;
}

void port_group_dots(int32_t *dots, const int8_t *xq, const int8_t *wq, int n, int d) {
    const int ng = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++)
        for (int g = 0; g < ng; g++)
            dots[(size_t)i * ng + g] = group_dot(xq + g * 32, wq + (size_t)i * n + g * 32);
}

/* src/utils.c:118-137.  The source reads sum += ((float)ival * w_scale) * x_scale; the
 * reference's -Ofast build reassociates the product and evaluates, for the groups in order and
 * without FMA contraction:
 *     sum = sum + (float)ival * (w_scale * x_scale)
 * (tests/test_oracle.py checks this bit for bit against the compiled reference). */
void port_matmul_q(float *out, const int8_t *xq, const float *xs, const int8_t *wq,
                   const float *ws, int n, int d) {
    const int ng = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const int8_t *w = wq + (size_t)i * n;
        const float *wsr = ws + (size_t)i * ng;
        float sum = 0.0f;
        for (int g = 0; g < ng; g++) {
            const int32_t ival = group_dot(xq + g * 32, w + g * 32);
            const float scale = wsr[g] * xs[g];
            sum = sum + (float)ival * scale;
        }
        out[i] = sum;
    }
}

/* matmul_Q8_0 (src/utils.c:106-138): quantise x (src/utils.c:107 -> src/tensor.c:199), then GEMV. */
void port_matmul(float *out, const float *x, const int8_t *wq, const float *ws, int n, int d) {
    int8_t *xq = malloc((size_t)n);
    float *xs = malloc((size_t)n / 32 * sizeof(float));
    port_quant_f32(x, (size_t)n, xq, xs);
    port_matmul_q(out, xq, xs, wq, ws, n, d);
    free(xq);
    free(xs);
}

/* rmsnorm (src/utils.c:59-76): ss = sum x^2; ss /= n; ss += 1e-5f; ss = 1/sqrtf(ss);
 * o = w * (ss * x).  eps is hard-coded in the reference (src/utils.c:70).
 *
 * The reference's -Ofast build vectorises the sum of squares over 8 lanes (lane k accumulates
 * x[8i+k]^2 in order, multiply then add), folds the lanes as ((s0+s4)+(s2+s6))+((s1+s5)+(s3+s7)),
 * and computes the output as (w*x)*ss; this restatement follows that order for n % 8 == 0 (every
 * model dimension here).  It computes 1/sqrtf exactly rounded, whereas the compiled reference
 * uses the CPU's rsqrt approximation plus one Newton step, so the scale can differ in the last
 * bit. */
void port_rmsnorm(float *o, const float *x, const float *w, int n) {
    float ss;
    if (n % 8 == 0) {
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < n; j += 8)
            for (int k = 0; k < 8; k++) lane[k] = lane[k] + x[j + k] * x[j + k];
        ss = ((lane[0] + lane[4]) + (lane[2] + lane[6])) + ((lane[1] + lane[5]) + (lane[3] + lane[7]));
    } else {
        ss = 0.0f;
        for (int j = 0; j < n; j++) ss = ss + x[j] * x[j];
    }
    ss = ss / (float)n;
    ss = ss + 1e-5f;
    ss = 1.0f / sqrtf(ss);
    for (int j = 0; j < n; j++) o[j] = (w[j] * x[j]) * ss;
}

/* softmax_f32 (src/utils.c:39-57). */
void port_softmax(float *x, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - max_val);
        sum = sum + x[i];
    }
    for (int i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* sample_argmax (src/sampler.c:6-17): strict '>' so the first maximum wins. */
int port_argmax(const float *x, int n) {
    int best = 0;
    float bv = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > bv) { best = i; bv = x[i]; }
    return best;
}

/* src/transformer.c:90-95: head_dim = 2j; freq = 1/powf(10000, head_dim/(float)hs);
 * val = pos * freq; (cosf(val), sinf(val)).  theta = 10000 is hard-coded in the reference. */
void port_rope_coeffs(int pos, int head_size, float *cs) {
    for (int j = 0; j < head_size / 2; j++) {
        const int head_dim = j * 2;
        const float freq = 1.0f / powf(10000.0f, (float)head_dim / (float)head_size);
        const float val = (float)pos * freq;
        cs[2 * j] = cosf(val);
        cs[2 * j + 1] = sinf(val);
    }
}

/* ---- sampler with temperature (src/sampler.c:20-131) ---- */

/* xorshift64* (src/sampler.c:96-102) and its [0,1) float (src/sampler.c:104-106). */
static unsigned int xs_u32(unsigned long long *st) {
    *st ^= *st >> 12;
    *st ^= *st << 25;
    *st ^= *st >> 27;
    return (unsigned int)((*st * 0x2545F4914F6CDD1Dull) >> 32);
}
static float xs_f32(unsigned long long *st) { return (float)(xs_u32(st) >> 8) / 16777216.0f; }

typedef struct { float prob; int index; } PortProbIndex;

static int cmp_prob_desc(const void *a, const void *b) {
    const PortProbIndex *x = a, *y = b;
    if (x->prob > y->prob) return -1;
    if (x->prob < y->prob) return 1;
    return 0;
}

int port_sample(float *logits, int n, float temperature, float topp, unsigned long long *rng) {
    if (temperature == 0.0f) return port_argmax(logits, n);
    for (int i = 0; i < n; i++) logits[i] = logits[i] / temperature;      /* sampler.c:116 */
    port_softmax(logits, n);                                               /* sampler.c:118 */
    const float coin = xs_f32(rng);                                        /* sampler.c:120 */
    if (topp <= 0 || topp >= 1) {                                          /* sample_mult, sampler.c:19-29 */
        float cdf = 0.0f;
        for (int i = 0; i < n; i++) {
            cdf = cdf + logits[i];
            if (coin < cdf) return i;
        }
        return n - 1;
    }
    /* sample_topp (sampler.c:38-86): drop candidates below (1-topp)/(n-1), sort descending,
     * truncate where the cumulative probability first exceeds topp, sample the truncated list. */
    PortProbIndex *pi = malloc((size_t)n * sizeof(PortProbIndex));
    int n0 = 0;
    const float cutoff = (1.0f - topp) / (float)(n - 1);
    for (int i = 0; i < n; i++)
        if (logits[i] >= cutoff) { pi[n0].index = i; pi[n0].prob = logits[i]; n0++; }
    qsort(pi, (size_t)n0, sizeof(PortProbIndex), cmp_prob_desc);
    float cum = 0.0f;
    int last = n0 - 1;
    for (int i = 0; i < n0; i++) {
        cum = cum + pi[i].prob;
        if (cum > topp) { last = i; break; }
    }
    const float r = coin * cum;
    float cdf = 0.0f;
    int result = pi[last].index;
    for (int i = 0; i <= last; i++) {
        cdf = cdf + pi[i].prob;
        if (r < cdf) { result = pi[i].index; break; }
    }
    free(pi);
    return result;
}

/* ---- whole-model forward (src/transformer.c:55-239) ---- */

typedef struct { const int8_t *q; const float *s; } PQ8;

typedef struct {
    const float *rms_att, *rms_ffn;
    PQ8 wq, wk, wv, wo, w1, w2, w3;
} PortLayer;

struct PortModel {
    int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len;
    int kv_f32;
    PQ8 emb, wcls;
    const float *rms_final;
    PortLayer *layers;
    /* run state (src/transformer.c:13-30) */
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
    void *key_cache, *value_cache; /* [layer][seq][kv_dim], bf16 or f32 */
    /* checkpoint recorder of port_forward_dump (NULL: off): the same checkpoints as the hooked
     * reference build (oracle/ref_hooks.c) */
    float *rec_x, *rec_in, *rec_s;
    int8_t *rec_q;
    int rec_nx;
    size_t rec_off;
};

/* Checkpoints (test infrastructure): the input of every rmsnorm (the residual stream), and the fp32
 * input plus Q8_0 form of the activation each distinct matmul input is quantised to. */
static void rec_x(PortModel *m, const float *x) {
    if (!m->rec_x) return;
    memcpy(m->rec_x + (size_t)m->rec_nx * m->dim, x, (size_t)m->dim * sizeof(float));
    m->rec_nx++;
}
static void rec_act(PortModel *m, const float *in, int n) {
    if (!m->rec_x) return;
    memcpy(m->rec_in + m->rec_off, in, (size_t)n * sizeof(float));
    port_quant_f32(in, (size_t)n, m->rec_q + m->rec_off, m->rec_s + m->rec_off / 32);
    m->rec_off += (size_t)n;
}

PortModel *port_model_create(const int *cfg, int kv_f32) {
    PortModel *m = calloc(1, sizeof(PortModel));
    m->dim = cfg[0]; m->hidden = cfg[1]; m->n_layers = cfg[2]; m->n_heads = cfg[3];
    m->n_kv_heads = cfg[4]; m->vocab = cfg[5]; m->seq_len = cfg[6];
    m->kv_f32 = kv_f32;
    const int kv_dim = m->dim * m->n_kv_heads / m->n_heads;
    m->layers = calloc((size_t)m->n_layers, sizeof(PortLayer));
    m->x = calloc((size_t)m->dim, 4); m->xb = calloc((size_t)m->dim, 4);
    m->xb2 = calloc((size_t)m->dim, 4); m->q = calloc((size_t)m->dim, 4);
    m->hb = calloc((size_t)m->hidden, 4); m->hb2 = calloc((size_t)m->hidden, 4);
    m->k = calloc((size_t)kv_dim, 4); m->v = calloc((size_t)kv_dim, 4);
    m->att = calloc((size_t)m->n_heads * (size_t)m->seq_len, 4);
    m->logits = calloc((size_t)m->vocab, 4);
    const size_t kv_elems = (size_t)m->n_layers * (size_t)m->seq_len * (size_t)kv_dim;
    const size_t esz = kv_f32 ? 4 : 2;
    m->key_cache = calloc(kv_elems, esz);
    m->value_cache = calloc(kv_elems, esz);
    return m;
}

void port_model_destroy(PortModel *m) {
    if (!m) return;
    free(m->layers); free(m->x); free(m->xb); free(m->xb2); free(m->q); free(m->hb);
    free(m->hb2); free(m->k); free(m->v); free(m->att); free(m->logits);
    free(m->key_cache); free(m->value_cache);
    free(m);
}

void port_model_set(PortModel *m, int which, int layer, const void *data, const float *scale) {
    PQ8 w = { (const int8_t *)data, scale };
    PortLayer *L = (layer >= 0 && layer < m->n_layers) ? &m->layers[layer] : NULL;
    switch (which) {
    case PW_EMB: m->emb = w; break;
    case PW_RMS_FINAL: m->rms_final = data; break;
    case PW_WCLS: m->wcls = w; break;
    case PW_RMS_ATT: if (L) L->rms_att = data; break;
    case PW_WQ: if (L) L->wq = w; break;
    case PW_WK: if (L) L->wk = w; break;
    case PW_WV: if (L) L->wv = w; break;
    case PW_WO: if (L) L->wo = w; break;
    case PW_RMS_FFN: if (L) L->rms_ffn = data; break;
    case PW_W1: if (L) L->w1 = w; break;
    case PW_W2: if (L) L->w2 = w; break;
    case PW_W3: if (L) L->w3 = w; break;
    default: break;
    }
}

static inline float kv_read(const PortModel *m, const void *cache, size_t idx) {
    return m->kv_f32 ? ((const float *)cache)[idx] : bf16_bits_to_f32(((const uint16_t *)cache)[idx]);
}

static inline void kv_write(const PortModel *m, void *cache, size_t idx, float v) {
    if (m->kv_f32) ((float *)cache)[idx] = v;
    else ((uint16_t *)cache)[idx] = f32_to_bf16_trunc(v);
}

void port_forward(PortModel *m, int token, int pos, float *logits, float *xdump) {
    const int dim = m->dim, hidden = m->hidden;
    const int kv_dim = dim * m->n_kv_heads / m->n_heads;
    const int kv_mul = m->n_heads / m->n_kv_heads;
    const int hs = dim / m->n_heads;
    float *x = m->x;

    /* embedding row dequant (src/transformer.c:69) */
    port_dequant(m->emb.q + (size_t)token * dim, m->emb.s + (size_t)token * dim / 32, (size_t)dim, x);

    float *cs = malloc((size_t)hs * sizeof(float));
    port_rope_coeffs(pos, hs, cs);

    for (int l = 0; l < m->n_layers; l++) {
        const PortLayer *L = &m->layers[l];
        rec_x(m, x);
        port_rmsnorm(m->xb, x, L->rms_att, dim);                               /* :77 */
        rec_act(m, m->xb, dim);
        const size_t loff = (size_t)l * m->seq_len * kv_dim;                   /* :80 */
        port_matmul(m->q, m->xb, L->wq.q, L->wq.s, dim, dim);                  /* :83-85 */
        port_matmul(m->k, m->xb, L->wk.q, L->wk.s, dim, kv_dim);
        port_matmul(m->v, m->xb, L->wv.q, L->wv.s, dim, kv_dim);

        /* HF rotate-half RoPE (src/transformer.c:87-119): pairs (j, j + hs/2) per head; keys
         * are rotated where the pair lies inside kv_dim.  The reference's -Ofast build contracts
         * the rotation into fused multiply-adds: a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c). */
        for (int i = 0; i < m->n_heads; i++) {
            for (int j = 0; j < hs / 2; j++) {
                const float fcr = cs[2 * j], fci = cs[2 * j + 1];
                const int i1 = i * hs + j, i2 = i * hs + j + hs / 2;
                const float q0 = m->q[i1], q1 = m->q[i2];
                m->q[i1] = fmaf(q0, fcr, -(q1 * fci));
                m->q[i2] = fmaf(q0, fci, q1 * fcr);
                if (i2 < kv_dim) {
                    const float k0 = m->k[i1], k1 = m->k[i2];
                    m->k[i1] = fmaf(k0, fcr, -(k1 * fci));
                    m->k[i2] = fmaf(k0, fci, k1 * fcr);
                }
            }
        }

        /* KV-cache write at [l][pos] (src/transformer.c:145-146) */
        for (int i = 0; i < kv_dim; i++) {
            kv_write(m, m->key_cache, loff + (size_t)pos * kv_dim + i, m->k[i]);
            kv_write(m, m->value_cache, loff + (size_t)pos * kv_dim + i, m->v[i]);
        }

        /* attention over t <= pos (src/transformer.c:149-193) */
        const float sq = sqrtf((float)hs);
        #pragma omp parallel for schedule(static)
        for (int h = 0; h < m->n_heads; h++) {
            const float *qh = m->q + h * hs;
            float *att = m->att + (size_t)h * m->seq_len;
            const size_t hoff = (size_t)(h / kv_mul) * hs;
            for (int t = 0; t <= pos; t++) {
                const size_t base = loff + (size_t)t * kv_dim + hoff;
                float score = 0.0f;
                for (int i = 0; i < hs; i++) score = score + qh[i] * kv_read(m, m->key_cache, base + i);
                att[t] = score / sq;
            }
            port_softmax(att, pos + 1);
            float *xbh = m->xb + h * hs;
            memset(xbh, 0, (size_t)hs * sizeof(float));
            for (int t = 0; t <= pos; t++) {
                const size_t base = loff + (size_t)t * kv_dim + hoff;
                const float a = att[t];
                for (int i = 0; i < hs; i++) xbh[i] = xbh[i] + a * kv_read(m, m->value_cache, base + i);
            }
        }

        rec_act(m, m->xb, dim);
        port_matmul(m->xb2, m->xb, L->wo.q, L->wo.s, dim, dim);               /* :196 */
        for (int i = 0; i < dim; i++) x[i] = x[i] + m->xb2[i];                 /* :199-201 */

        rec_x(m, x);
        port_rmsnorm(m->xb, x, L->rms_ffn, dim);                               /* :204 */
        rec_act(m, m->xb, dim);
        port_matmul(m->hb, m->xb, L->w1.q, L->w1.s, dim, hidden);             /* :208 */
        port_matmul(m->hb2, m->xb, L->w3.q, L->w3.s, dim, hidden);            /* :209 */
        for (int i = 0; i < hidden; i++) {                                     /* :212-222 */
            float val = m->hb[i];
            val = val * (1.0f / (1.0f + expf(-val)));
            val = val * m->hb2[i];
            m->hb[i] = val;
        }
        rec_act(m, m->hb, hidden);
        port_matmul(m->xb, m->hb, L->w2.q, L->w2.s, hidden, dim);             /* :225 */
        for (int i = 0; i < dim; i++) x[i] = x[i] + m->xb[i];                  /* :228-230 */

        if (xdump) memcpy(xdump + (size_t)l * dim, x, (size_t)dim * sizeof(float));
    }

    rec_x(m, x);
    port_rmsnorm(x, x, m->rms_final, dim);                                     /* :234 */
    rec_act(m, x, dim);
    port_matmul(m->logits, x, m->wcls.q, m->wcls.s, dim, m->vocab);            /* :237 */
    memcpy(logits, m->logits, (size_t)m->vocab * sizeof(float));
    free(cs);
}

/* The greedy loop of generate (src/bin/localinfer.c:42-99) on token ids: force prompt tokens,
 * then argmax; stop when the next token is 1. */
int port_generate(PortModel *m, const int *prompt, int n_prompt, int steps, int *out) {
    int token = prompt[0], pos = 0, n_out = 0;
    float *logits = malloc((size_t)m->vocab * sizeof(float));
    while (pos < steps) {
        port_forward(m, token, pos, logits, NULL);
        int next;
        if (pos < n_prompt - 1) {
            next = prompt[pos + 1];
        } else {
            next = port_argmax(logits, m->vocab);
            out[n_out++] = next;
        }
        pos++;
        if (next == 1) break;
        token = next;
    }
    free(logits);
    return n_out;
}

/* port_forward with the checkpoints recorded (same layout as oref_forward_dump in ref_hooks.c):
 * xres [2L+1][dim]; per layer the activations of wq, wo, w1, w2 and then wcls's, concatenated in
 * ain / aq (n each) and as (n/32 each). */
void port_forward_dump(PortModel *m, int token, int pos, float *logits, float *xres, float *ain, int8_t *aq,
                       float *as) {
    m->rec_x = xres; m->rec_in = ain; m->rec_q = aq; m->rec_s = as;
    m->rec_nx = 0; m->rec_off = 0;
    port_forward(m, token, pos, logits, NULL);
    m->rec_x = NULL; m->rec_in = NULL; m->rec_q = NULL; m->rec_s = NULL;
}

/* KV-cache rows [pos0, pos0+n) of one layer in the cache's own element type ([n][kv_dim]). */
void port_kv_rows(const PortModel *m, int layer, int pos0, int n, void *k, void *v) {
    const size_t kv_dim = (size_t)m->dim * m->n_kv_heads / m->n_heads;
    const size_t esz = m->kv_f32 ? 4 : 2;
    const size_t off = ((size_t)layer * m->seq_len + pos0) * kv_dim * esz;
    memcpy(k, (const uint8_t *)m->key_cache + off, kv_dim * (size_t)n * esz);
    memcpy(v, (const uint8_t *)m->value_cache + off, kv_dim * (size_t)n * esz);
}

/* Overwrite KV-cache rows [pos0, pos0+n) of one layer with rows of the cache's element type. */
void port_kv_write(PortModel *m, int layer, int pos0, int n, const void *k, const void *v) {
    const size_t kv_dim = (size_t)m->dim * m->n_kv_heads / m->n_heads;
    const size_t esz = m->kv_f32 ? 4 : 2;
    const size_t off = ((size_t)layer * m->seq_len + pos0) * kv_dim * esz;
    memcpy((uint8_t *)m->key_cache + off, k, kv_dim * (size_t)n * esz);
    memcpy((uint8_t *)m->value_cache + off, v, kv_dim * (size_t)n * esz);
}
