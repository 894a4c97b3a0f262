/*
 * host_internal.h -- shared pieces of the reference-API host library (tensor.c, utils.c,
 * safetensors.c, transformer.c, sampler.c, tokenizer.c): a small JSON reader, the exit-on-error
 * helpers that give these entry points the reference's failure behaviour (message on stderr, then
 * exit(EXIT_FAILURE)), and device staging buffers for the GPU-backed conversions.
 */
#ifndef DIOLKOS_HOST_INTERNAL_H
#define DIOLKOS_HOST_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "tensor.h"

/* ---- JSON ------------------------------------------------------------------------------------ */
typedef enum { JS_NULL, JS_BOOL, JS_NUM, JS_STR, JS_ARR, JS_OBJ } js_kind;

typedef struct js_node {
    js_kind kind;
    double num;             /* JS_NUM, JS_BOOL (0 / 1)                          */
    char *str;              /* JS_STR: decoded UTF-8, NUL-terminated            */
    int n;                  /* JS_ARR / JS_OBJ: number of members                */
    struct js_node *kids;   /* JS_ARR / JS_OBJ: member values, in document order */
    char **keys;            /* JS_OBJ: member names, in document order           */
} js_node;

/* Parse text[0..len) as one JSON value (trailing whitespace allowed).  NULL on a syntax error, with
 * a message in err. */
js_node *js_parse(const char *text, size_t len, char *err, size_t err_len);
void js_free(js_node *v);
/* The member `key` of an object (the first one, if repeated), or NULL. */
const js_node *js_get(const js_node *obj, const char *key);
/* Numeric value of member `key`, or `dflt` when it is absent or not a number. */
double js_num(const js_node *obj, const char *key, double dflt);

/* ---- errors ---------------------------------------------------------------------------------- */
/* Print "diolkos: <what>: <dk_last_error()>" and exit(EXIT_FAILURE) when status != 0. */
void host_check(int status, const char *what);
/* Print the CUDA error and exit(EXIT_FAILURE) when e != 0 (e is a cudaError_t). */
void host_check_cuda(int e, const char *what);
/* malloc / calloc that exit on failure. */
void *host_malloc(size_t n);
void *host_calloc(size_t n, size_t size);

/* ---- device staging -------------------------------------------------------------------------- */
/* A growable device buffer owned by the caller's static state, on the device that was current when
 * it was allocated. */
typedef struct {
    void *ptr;
    size_t bytes;
    int device;
} dev_buf;
/* Make b at least `bytes` long on the current device (contents are not kept; a buffer on another
 * device is released and replaced); exits on failure. */
void *dev_reserve(dev_buf *b, size_t bytes);

/* Drop the GPU copy utils.c keeps of a matrix used with matmul() (called by tensor_destroy). */
void utils_forget_tensor(const Tensor *t);

/* load_safetensors allocates a Model inside this larger block, so that the GPU model built from it
 * can be found from Transformer.safetensors while Transformer keeps the reference's layout. */
struct Model;
struct dk_model;
struct dk_model **model_engine_slot(struct Model *m);
int *model_tp_slot(struct Model *m);  /* {rank, world} of the engine */
struct Model *model_ext_alloc(void);

#endif
