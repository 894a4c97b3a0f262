/*
 * transformer.c -- the reference's model API (src/transformer.c:13-53 and forward, :55-239) over the
 * B200 decode engine.
 *
 * build_transformer_from_safetensors loads the directory with load_safetensors (host Q8_0 tensors,
 * cached exactly like the reference), creates the engine on the current CUDA device with the
 * reference's bf16 KV cache, hands it every weight and captures the per-token CUDA graph.  forward
 * runs one step on the GPU and copies the logits into the host RunState, so callers read them the
 * way they read the reference's.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "diolkos.h"
#include "host_internal.h"
#include "safetensors.h"
#include "tensor.h"
#include "transformer.h"

void malloc_run_state(RunState *s, Config *p) {
    memset(s, 0, sizeof *s);
    s->logits = tensor_create((size_t)p->vocab_size, F32);
}

static void set_q8(dk_model *m, int which, int layer, Tensor *t) {
    if (t->type != Q8_0) {
        fprintf(stderr, "diolkos: weight %d (layer %d) is %s, expected Q8_0\n", which, layer, quant_t_to_string(t->type));
        exit(EXIT_FAILURE);
    }
    host_check(dk_model_set_weight(m, which, layer, t->data, t->scale), "set weight");
}

static void set_f32(dk_model *m, int which, int layer, Tensor *t) {
    host_check(dk_model_set_weight(m, which, layer, data_f32(t), NULL), "set weight");
}

void build_transformer_from_safetensors(Transformer *t, const char *model_path) {
    Model *st = load_safetensors(model_path);
    if (!st) {
        fprintf(stderr, "Failed to load safetensors model from %s\n", model_path);
        exit(EXIT_FAILURE);
    }
    t->config = *st->config;
    t->safetensors = st;
    malloc_run_state(&t->state, &t->config);

    const Config *c = &t->config;
    int device = 0;
    host_check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    const int cfg[7] = {c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads, c->vocab_size, c->seq_len};
    t->engine = dk_model_create(cfg, DK_KV_BF16, device, 0, 1);
    if (!t->engine) host_check(DK_ERR_INVALID, "create the model");
    set_q8(t->engine, DK_W_EMB, -1, st->token_embedding_table);
    set_f32(t->engine, DK_W_RMS_FINAL, -1, st->rms_final_weight);
    set_q8(t->engine, DK_W_WCLS, -1, st->wcls);
    for (int l = 0; l < c->n_layers; ++l) {
        Layer *L = &st->layers[l];
        set_f32(t->engine, DK_W_RMS_ATT, l, L->rms_att_weight);
        set_q8(t->engine, DK_W_WQ, l, L->wq);
        set_q8(t->engine, DK_W_WK, l, L->wk);
        set_q8(t->engine, DK_W_WV, l, L->wv);
        set_q8(t->engine, DK_W_WO, l, L->wo);
        set_f32(t->engine, DK_W_RMS_FFN, l, L->rms_ffn_weight);
        set_q8(t->engine, DK_W_W1, l, L->w1);
        set_q8(t->engine, DK_W_W2, l, L->w2);
        set_q8(t->engine, DK_W_W3, l, L->w3);
    }
    host_check(dk_model_finalize(t->engine), "finalize the model");
    fprintf(stderr,
            "Transformer config from safetensors: dim=%d, hidden_dim=%d, n_layers=%d, n_heads=%d, n_kv_heads=%d, "
            "vocab_size=%d, seq_len=%d\n",
            c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads, c->vocab_size, c->seq_len);
}

Tensor *forward(Transformer *transformer, int token, int pos) {
    host_check(dk_model_forward(transformer->engine, token, pos, data_f32(transformer->state.logits)), "forward");
    return transformer->state.logits;
}

void free_transformer(Transformer *t) {
    if (t->engine) dk_model_destroy(t->engine);
    t->engine = NULL;
    tensor_destroy(t->state.logits);
    t->state.logits = NULL;
}
