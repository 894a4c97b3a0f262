/*
 * transformer.h -- the reference's model API (src/transformer.h) served by the B200 engine.
 *
 * build_transformer_from_safetensors loads a HF LLaMA-2 directory exactly like the reference
 * (config.json, *.safetensors, the Q8_0 cache under ./cache/<model>/), then moves the whole model to
 * the current CUDA device (dk_model_* in diolkos.h).  forward() runs one decode step there as one
 * CUDA graph and returns the logits in a HOST tensor, as the reference does.
 */
#ifndef DIOLKOS_TRANSFORMER_H
#define DIOLKOS_TRANSFORMER_H

#include <stddef.h>
#include <stdint.h>

#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct Model Model;

typedef struct {
    int dim;        /* transformer dimension                              */
    int hidden_dim; /* FFN dimension                                      */
    int n_layers;
    int n_heads;    /* query heads                                        */
    int n_kv_heads; /* key/value heads (fewer than n_heads with GQA)      */
    int vocab_size;
    int seq_len;    /* maximum sequence length                            */
} Config;

/* The reference keeps every activation here.  On the B200 they live on the device inside the
 * engine: `logits` (host F32, vocab_size values) is written by each forward; x .. att, k, v are host
 * tensors of the reference's sizes that the GPU path does not write; key_cache / value_cache
 * describe the size of the bf16 KV cache (held in HBM) and have no host data. */
typedef struct {
    Tensor *x, *xb, *xb2, *hb, *hb2, *q, *att, *logits;
    Tensor *key_cache, *value_cache;
    Tensor *k, *v;
} RunState;

/* Same layout as the reference's, so callers may allocate it themselves (as localinfer does, on the
 * stack): the GPU model is reached through `safetensors`, which this library allocates. */
typedef struct Transformer {
    Config config;
    RunState state;
    Model *safetensors;        /* the host weights as loaded (and cached) */
} Transformer;

/* Allocate the host-side state (the logits tensor) for a model of this shape. */
void malloc_run_state(RunState *s, Config *p);
/* Load `model_path` (a directory) and build the GPU model on the current CUDA device, with the
 * reference's bf16 KV cache.  Exits with a message on failure, like the reference. */
void build_transformer_from_safetensors(Transformer *t, const char *model_path);
/* One decode step at `pos` with input `token`; returns the host logits (t->state.logits). */
Tensor *forward(Transformer *transformer, int token, int pos);
/* Tensor-parallel build: the reference's client/worker split (src/bin/client.c: heads and weight rows
 * spread over workers), here over the GPUs of one box, one process per GPU.  Rank `rank` of `world`
 * loads the model like build_transformer_from_safetensors and creates its shard on CUDA device
 * `device`; `handle` receives DK_COMM_HANDLE_BYTES (diolkos.h) bytes to hand to every other rank (any
 * transport).  build_transformer_tp_connect, given all ranks' handles in rank order, connects the
 * ranks, uploads this rank's slices of the weights and captures the step.  Every rank must then run
 * the same forward() calls in the same order; each fills only its own classifier rows of
 * t->state.logits.  Exits with a message on failure. */
void build_transformer_tp(Transformer *t, const char *model_path, int rank, int world, int device, void *handle);
void build_transformer_tp_connect(Transformer *t, const void *handles);
/* First and one-past-last vocabulary rows this rank's forward() writes ([0, vocab) with one rank). */
void transformer_logit_rows(Transformer *t, int *begin, int *end);
/* The GPU model behind a built transformer (diolkos.h: dk_model_*), for callers that want the
 * engine's own entry points (dk_model_generate, dk_model_weight_bytes, ...); NULL before
 * build_transformer_from_safetensors. */
struct dk_model *transformer_engine(Transformer *t);
/* The forward() calls of positions 0 .. n-1 with tokens[0 .. n-1], batched (no counterpart in the
 * reference, whose generate loop forwards prompt tokens one by one, src/bin/localinfer.c:60-73): one
 * prefill on the GPU's tensor cores that leaves the KV cache exactly as those forward() calls would;
 * no logits.  forward(tokens[n], n) continues from there.  Tensor parallel: every rank calls it.
 * Returns 0, or the DK_ERR_* code (with the message on stderr) when the engine cannot prefill. */
int transformer_prefill(Transformer *t, const int *tokens, int n);
/* Release the GPU model and the host RunState tensors (no counterpart in the reference, which never
 * frees); the host weights in t->safetensors stay. */
void free_transformer(Transformer *t);

#ifdef __cplusplus
}
#endif
#endif
