/*
 * port.h -- CPU restatement of the reference's per-token decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the oracle that the CUDA path is checked against; only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.  It is pinned
 * against the reference itself (oracle/_ref, built from the unmodified reference sources) and
 * against the committed fixtures under tests/golden/.
 *
 * Every function names the reference file:line it restates (paths relative to the reference
 * project root).  Arithmetic is spelled out operation by operation and the file is compiled with
 * -ffp-contract=off -fno-fast-math, so the result does not depend on compiler flags.
 */
#ifndef DIOLKOS_ORACLE_PORT_H
#define DIOLKOS_ORACLE_PORT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight quantiser used at load time (src/tensor.c:312-344). */
void port_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s);
/* Activation quantiser used before every matmul (src/tensor.c:199-228). */
void port_quant_f32(const float *x, size_t n, int8_t *q, float *s);
/* Dequantise a Q8_0 slice (src/tensor.c:245-265). */
void port_dequant(const int8_t *q, const float *s, size_t n, float *out);
/* matmul_Q8_0 (src/utils.c:106-138): out[d] = W[d x n] * quant(x[n]). */
void port_matmul(float *out, const float *x, const int8_t *wq, const float *ws, int n, int d);
/* Same GEMV on an already-quantised activation. */
void port_matmul_q(float *out, const int8_t *xq, const float *xs, const int8_t *wq,
                   const float *ws, int n, int d);
/* The exact int32 group dots of matmul_Q8_0 (src/utils.c:122-127): dots[d][n/32]. */
void port_group_dots(int32_t *dots, const int8_t *xq, const int8_t *wq, int n, int d);
/* rmsnorm (src/utils.c:59-76). */
void port_rmsnorm(float *o, const float *x, const float *w, int n);
/* softmax_f32 (src/utils.c:39-57), in place. */
void port_softmax(float *x, int n);
/* sample_argmax (src/sampler.c:6-17). */
int port_argmax(const float *x, int n);
/* The HF rotate-half RoPE coefficient table for one position (src/transformer.c:90-95):
 * cs[2*j] = cosf(pos*freq_j), cs[2*j+1] = sinf(pos*freq_j), j < head_size/2. */
void port_rope_coeffs(int pos, int head_size, float *cs);
/* sample (src/sampler.c:108-131) with temperature > 0: softmax + xorshift coin + top-p/mult. */
int port_sample(float *logits, int n, float temperature, float topp, unsigned long long *rng);

/* ---- whole-model restatement of forward (src/transformer.c:55-239) ---- */
typedef struct PortModel PortModel;

enum PortWeight {
    PW_EMB = 0,      /* model.embed_tokens.weight  Q8_0 [V x d]   */
    PW_RMS_FINAL,    /* model.norm.weight          F32  [d]       */
    PW_WCLS,         /* lm_head.weight             Q8_0 [V x d]   */
    PW_RMS_ATT,      /* per layer: input_layernorm F32 [d]        */
    PW_WQ, PW_WK, PW_WV, PW_WO,
    PW_RMS_FFN,
    PW_W1, PW_W2, PW_W3,
};

/* cfg = {dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len}.
 * kv_f32 = 0 keeps the reference's bf16-truncating KV cache (src/transformer.c:25-26, :145-146);
 * kv_f32 = 1 stores the KV cache in fp32. */
PortModel *port_model_create(const int *cfg, int kv_f32);
void port_model_destroy(PortModel *m);
/* Register a weight (the pointers are borrowed and must stay valid). scale == NULL for F32. */
void port_model_set(PortModel *m, int which, int layer, const void *data, const float *scale);
/* One decode step; writes logits[vocab]; if xdump != NULL, writes the residual stream after each
 * layer to xdump[l*dim .. (l+1)*dim). */
void port_forward(PortModel *m, int token, int pos, float *logits, float *xdump);
/* port_forward recording per-layer checkpoints: xres[2L+1][dim] = the input of every rmsnorm (the
 * residual stream; src/transformer.c:76, :204, :234); per layer the fp32 input and Q8_0 form of the
 * activations of wq (:83), wo (:196), w1 (:208), w2 (:225), then of wcls (:237), concatenated in
 * ain / aq and as. */
void port_forward_dump(PortModel *m, int token, int pos, float *logits, float *xres, float *ain, int8_t *aq,
                       float *as);
/* KV-cache rows [pos0, pos0+n) of one layer, [n][kv_dim] in the cache's element type. */
void port_kv_rows(const PortModel *m, int layer, int pos0, int n, void *k, void *v);
/* Overwrite KV-cache rows [pos0, pos0+n) of one layer with rows of the cache's element type. */
void port_kv_write(PortModel *m, int layer, int pos0, int n, const void *k, const void *v);
/* Greedy generate loop (src/bin/localinfer.c:42-99) on token ids; returns #generated tokens. */
int port_generate(PortModel *m, const int *prompt, int n_prompt, int steps, int *out);

#ifdef __cplusplus
}
#endif
#endif
