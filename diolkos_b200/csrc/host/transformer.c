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

/* The reference's RunState sizes (src/transformer.c:13-30).  Only logits is written on this path;
 * the KV-cache tensors are descriptors of the bf16 cache the engine keeps in HBM (no host data). */
void malloc_run_state(RunState *s, Config *p) {
    const size_t kv_dim = (size_t)p->dim * (size_t)p->n_kv_heads / (size_t)p->n_heads;
    memset(s, 0, sizeof *s);
    s->x = tensor_create((size_t)p->dim, F32);
    s->xb = tensor_create((size_t)p->dim, F32);
    s->xb2 = tensor_create((size_t)p->dim, F32);
    s->hb = tensor_create((size_t)p->hidden_dim, F32);
    s->hb2 = tensor_create((size_t)p->hidden_dim, F32);
    s->q = tensor_create((size_t)p->dim, F32);
    s->att = tensor_create((size_t)p->n_heads * (size_t)p->seq_len, F32);
    s->logits = tensor_create((size_t)p->vocab_size, F32);
    Tensor *kv[2];
    for (int i = 0; i < 2; ++i) {
        kv[i] = host_calloc(1, sizeof(Tensor));
        kv[i]->type = BF16;
        kv[i]->dim = (size_t)p->n_layers * (size_t)p->seq_len * kv_dim;
        kv[i]->vdim = 1;
        kv[i]->hdim = kv[i]->dim;
    }
    s->key_cache = kv[0];
    s->value_cache = kv[1];
    s->k = tensor_create(kv_dim, F32);
    s->v = tensor_create(kv_dim, F32);
}

struct dk_model *transformer_engine(Transformer *t) {
    return t && t->safetensors ? *model_engine_slot(t->safetensors) : NULL;
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

static void transformer_tp_shape(Transformer *t, int *rank, int *world) {
    *rank = 0;
    *world = 1;
    if (t && t->safetensors) {
        const int *tp = model_tp_slot(t->safetensors);
        if (tp[1] > 0) {
            *rank = tp[0];
            *world = tp[1];
        }
    }
}

/* Load the model, size the state and create this rank's engine shard. */
static dk_model *create_engine(Transformer *t, const char *model_path, int rank, int world, int device) {
    Model *st = load_safetensors(model_path);
    if (!st) {
        fprintf(stderr, "Failed to load safetensors model from %s\n", model_path);
        exit(EXIT_FAILURE);
    }
    t->config = *st->config;
    t->safetensors = st;
    malloc_run_state(&t->state, &t->config);
    const Config *c = &t->config;
    const int cfg[7] = {c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads, c->vocab_size, c->seq_len};
    dk_model *g = dk_model_create(cfg, DK_KV_BF16, device, rank, world);
    if (!g) host_check(DK_ERR_INVALID, "create the model");
    *model_engine_slot(st) = g;
    model_tp_slot(st)[0] = rank;
    model_tp_slot(st)[1] = world;
    return g;
}

/* Hand every weight to the engine (it keeps this rank's slices) and capture the step. */
static void finish_engine(Transformer *t) {
    Model *st = t->safetensors;
    dk_model *g = *model_engine_slot(st);
    const Config *c = &t->config;
    set_q8(g, DK_W_EMB, -1, st->token_embedding_table);
    set_f32(g, DK_W_RMS_FINAL, -1, st->rms_final_weight);
    set_q8(g, DK_W_WCLS, -1, st->wcls);
    for (int l = 0; l < c->n_layers; ++l) {
        Layer *L = &st->layers[l];
        set_f32(g, DK_W_RMS_ATT, l, L->rms_att_weight);
        set_q8(g, DK_W_WQ, l, L->wq);
        set_q8(g, DK_W_WK, l, L->wk);
        set_q8(g, DK_W_WV, l, L->wv);
        set_q8(g, DK_W_WO, l, L->wo);
        set_f32(g, DK_W_RMS_FFN, l, L->rms_ffn_weight);
        set_q8(g, DK_W_W1, l, L->w1);
        set_q8(g, DK_W_W2, l, L->w2);
        set_q8(g, DK_W_W3, l, L->w3);
    }
    host_check(dk_model_finalize(g), "finalize the model");
    fprintf(stderr,
            "Transformer config from safetensors: dim=%d, hidden_dim=%d, n_layers=%d, n_heads=%d, n_kv_heads=%d, "
            "vocab_size=%d, seq_len=%d\n",
            c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads, c->vocab_size, c->seq_len);
}

void build_transformer_from_safetensors(Transformer *t, const char *model_path) {
    int device = 0;
    host_check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    create_engine(t, model_path, 0, 1, device);
    finish_engine(t);
}

void build_transformer_tp(Transformer *t, const char *model_path, int rank, int world, int device, void *handle) {
    if (world < 1 || rank < 0 || rank >= world) {
        fprintf(stderr, "build_transformer_tp: rank %d of %d\n", rank, world);
        exit(EXIT_FAILURE);
    }
    host_check_cuda(cudaSetDevice(device), "cudaSetDevice");
    dk_model *g = create_engine(t, model_path, rank, world, device);
    if (world > 1) host_check(dk_model_comm_handle(g, handle), "export the exchange area");
}

void build_transformer_tp_connect(Transformer *t, const void *handles) {
    dk_model *g = transformer_engine(t);
    if (!g) host_check(DK_ERR_STATE, "build_transformer_tp_connect: build_transformer_tp first");
    int rank = 0, world = 1;
    transformer_tp_shape(t, &rank, &world);
    if (world > 1) host_check(dk_model_comm_connect(g, handles), "connect the ranks");
    finish_engine(t);
}

void transformer_logit_rows(Transformer *t, int *begin, int *end) {
    int rank = 0, world = 1;
    transformer_tp_shape(t, &rank, &world);
    const int V = t->config.vocab_size, per = (V + world - 1) / world;
    const int b = rank * per, e = b + per < V ? b + per : V;
    if (begin) *begin = b;
    if (end) *end = e;
}

Tensor *forward(Transformer *transformer, int token, int pos) {
    dk_model *g = transformer_engine(transformer);
    if (!g) host_check(DK_ERR_STATE, "forward: the transformer was not built");
    host_check(dk_model_forward(g, token, pos, data_f32(transformer->state.logits)), "forward");
    return transformer->state.logits;
}

int transformer_prefill(Transformer *t, const int *tokens, int n) {
    dk_model *g = transformer_engine(t);
    if (!g) return DK_ERR_STATE;
    if (n <= 0) return DK_OK;
    int r = dk_model_set_tokens(g, tokens, n, n);
    if (!r) r = dk_model_prefill(g, 0, n);
    if (!r) r = dk_model_sync(g);
    if (!r) r = dk_model_device_error(g);
    if (r) fprintf(stderr, "transformer_prefill: %s (code 0x%x)\n", dk_last_error(), r);
    return r;
}

void free_transformer(Transformer *t) {
    dk_model *g = transformer_engine(t);
    if (g) dk_model_destroy(g);
    if (t->safetensors) *model_engine_slot(t->safetensors) = NULL;
    Tensor **all[] = {&t->state.x, &t->state.xb, &t->state.xb2, &t->state.hb, &t->state.hb2, &t->state.q,
                      &t->state.att, &t->state.logits, &t->state.key_cache, &t->state.value_cache, &t->state.k,
                      &t->state.v};
    for (size_t i = 0; i < sizeof all / sizeof all[0]; ++i) {
        tensor_destroy(*all[i]);
        *all[i] = NULL;
    }
}
