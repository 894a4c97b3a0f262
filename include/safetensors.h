/*
 * safetensors.h -- the reference's loader (src/safetensors.h): HF LLaMA-2 weights from a directory.
 *
 * load_safetensors reads config.json and every *.safetensors file in the directory (8-byte
 * little-endian header length, JSON header, raw tensor data), and returns the weights as HOST tensors:
 * norms as F32, every matrix and the embedding as Q8_0.  Like the reference it keeps a cache of the
 * converted tensors in ./cache/<directory basename>/<tensor name>-<Q8_0|F32>.tensor (int8 values then
 * fp32 scales for Q8_0), reads a tensor from there when the file exists and writes it otherwise; the
 * quantisation itself runs on the GPU and is bit-identical to the reference's.
 */
#ifndef DIOLKOS_SAFETENSORS_H
#define DIOLKOS_SAFETENSORS_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "tensor.h"
#include "transformer.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    Tensor *rms_att_weight; /* F32 [dim]               */
    Tensor *rms_ffn_weight; /* F32 [dim]               */
    Tensor *wq;             /* Q8_0 [dim x dim]        */
    Tensor *wk;             /* Q8_0 [kv_dim x dim]     */
    Tensor *wv;             /* Q8_0 [kv_dim x dim]     */
    Tensor *wo;             /* Q8_0 [dim x dim]        */
    Tensor *w1;             /* Q8_0 [hidden x dim]     */
    Tensor *w2;             /* Q8_0 [dim x hidden]     */
    Tensor *w3;             /* Q8_0 [hidden x dim]     */
} Layer;

typedef struct Model {
    Config *config;
    bool huggingface_rope;           /* always true: rotate-half RoPE    */
    Tensor *token_embedding_table;   /* Q8_0 [vocab x dim]               */
    Layer *layers;                   /* n_layers                         */
    Tensor *rms_final_weight;        /* F32 [dim]                        */
    Tensor *wcls;                    /* Q8_0 [vocab x dim] (lm_head)     */
} Model;

/* Load the model in directory `dir`; exits with a message if a required tensor is missing. */
Model *load_safetensors(const char *dir);

#ifdef __cplusplus
}
#endif
#endif
