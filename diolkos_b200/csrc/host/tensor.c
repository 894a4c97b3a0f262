/*
 * tensor.c -- the reference's Tensor container and conversions (src/tensor.c) for host tensors.
 *
 * Storage follows the reference: one buffer per tensor, Q8_0 scales right after the int8 values
 * (tensor_create, src/tensor.c:80-92).  Quantisation and dequantisation run on the current CUDA
 * device through the library's kernels (dk_quantize_*_q8_0, dk_dequantize_q8_0), in chunks, with
 * the reference's exact rounding; widening 16-bit floats to fp32 is an exact bit operation done
 * here.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <unistd.h>

#include <cuda_runtime_api.h>

#include "diolkos.h"
#include "host_internal.h"
#include "tensor.h"

/* Elements converted per device round trip: bounds the staging memory (64 Mi values). */
#define CONVERT_CHUNK ((size_t)1 << 26)

float bf16_to_float(uint16_t bf16) {
    const uint32_t bits = (uint32_t)bf16 << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

float f16_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const int e = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF, bits;
    if (e == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);  /* inf / NaN (payload kept) */
    } else if (e != 0) {
        bits = sign | ((uint32_t)(e - 15 + 127) << 23) | (mant << 13);
    } else if (mant == 0) {
        bits = sign;  /* +-0 */
    } else {
        /* subnormal half: value = mant * 2^-24; normalise so the leading one is bit 10 */
        int shift = 0;
        while (!(mant & 0x400)) { mant <<= 1; ++shift; }
        bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | ((mant & 0x3FF) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

int quant_size(quant_t type) {
    switch (type) {
        case F32: return 4;
        case F16: case BF16: return 2;
        case Q8_0: return 1;
        default:
            fprintf(stderr, "diolkos: quant_size: unsupported type %d\n", (int)type);
            exit(EXIT_FAILURE);
    }
}

int group_size(quant_t type) { return (type == Q8_0 || type == Q4_0) ? 32 : 1; }

const char *quant_t_to_string(quant_t type) {
    switch (type) {
        case F32: return "F32";
        case F16: return "F16";
        case BF16: return "BF16";
        case Q8_0: return "Q8_0";
        case Q4_0: return "Q4_0";
    }
    return "?";
}

size_t Tensor_storage_size(Tensor *t) {
    size_t bytes = t->dim * (size_t)quant_size(t->type);
    if (t->type == Q8_0) bytes += t->dim / 32 * sizeof(float);
    return bytes;
}

size_t tensor_memory(Tensor *t) {
    size_t bytes = t->dim * (size_t)quant_size(t->type);
    if (t->scale) bytes += t->dim / (size_t)group_size(t->type) * sizeof(float);
    return bytes;
}

Tensor *tensor_create(size_t size, quant_t type) {
    Tensor *t = host_calloc(1, sizeof(Tensor));
    t->type = type;
    t->dim = size;
    t->vdim = 1;
    t->hdim = size;
    /* 32-byte aligned like the reference's aligned_alloc; zero-filled. */
    const size_t bytes = (Tensor_storage_size(t) + 31) & ~(size_t)31;
    void *p = NULL;
    if (posix_memalign(&p, 64, bytes ? bytes : 64) != 0) {
        fprintf(stderr, "diolkos: tensor_create: out of host memory (%zu bytes)\n", bytes);
        exit(EXIT_FAILURE);
    }
    memset(p, 0, bytes);
    t->data = (TensorData *)p;
    if (type == Q8_0) t->scale = (float *)((uint8_t *)p + size);
    return t;
}

void tensor_destroy(Tensor *t) {
    if (!t) return;
    utils_forget_tensor(t);
    if (t->fd == -2) {  /* a view into a file mapping it does not own (safetensors.c) */
        free(t);
        return;
    }
    if (t->fd) {  /* mapped from a cache file (safetensors.c): fd > 0 is still open */
        munmap(t->data, Tensor_storage_size(t));
        if (t->fd > 0) close(t->fd);
    } else {
        free(t->data);
    }
    free(t);
}

float *data_f32(Tensor *t) {
    if (t->type != F32) {
        fprintf(stderr, "diolkos: data_f32 on a %s tensor\n", quant_t_to_string(t->type));
        exit(EXIT_FAILURE);
    }
    return (float *)t->data;
}

int8_t *data_i8(Tensor *t) {
    if (t->type != Q8_0) {
        fprintf(stderr, "diolkos: data_i8 on a %s tensor\n", quant_t_to_string(t->type));
        exit(EXIT_FAILURE);
    }
    return (int8_t *)t->data;
}

static dev_buf g_src, g_q, g_s;

/* F32 / F16 / BF16 -> Q8_0 on the GPU, chunk by chunk. */
static Tensor *quantize(Tensor *in) {
    if (in->dim % 32) return NULL;
    Tensor *out = tensor_create(in->dim, Q8_0);
    out->vdim = in->vdim;
    out->hdim = in->hdim;
    const size_t es = (size_t)quant_size(in->type);
    for (size_t at = 0; at < in->dim; at += CONVERT_CHUNK) {
        const size_t n = in->dim - at < CONVERT_CHUNK ? in->dim - at : CONVERT_CHUNK;
        void *src = dev_reserve(&g_src, CONVERT_CHUNK * 4);
        int8_t *q = dev_reserve(&g_q, CONVERT_CHUNK);
        float *s = dev_reserve(&g_s, CONVERT_CHUNK / 32 * sizeof(float));
        host_check_cuda(cudaMemcpy(src, (const uint8_t *)in->data + at * es, n * es, cudaMemcpyHostToDevice),
                        "convert: copy to device");
        int st;
        if (in->type == F32) st = dk_quantize_f32_q8_0(src, n, q, s, NULL);
        else if (in->type == BF16) st = dk_quantize_bf16_q8_0(src, n, q, s, NULL);
        else st = dk_quantize_f16_q8_0(src, n, q, s, NULL);
        host_check(st, "convert: quantise");
        host_check_cuda(cudaMemcpy(data_i8(out) + at, q, n, cudaMemcpyDeviceToHost), "convert: copy values back");
        host_check_cuda(cudaMemcpy(out->scale + at / 32, s, n / 32 * sizeof(float), cudaMemcpyDeviceToHost),
                        "convert: copy scales back");
    }
    return out;
}

/* Q8_0 -> F32 on the GPU (convert_q8_f32, src/tensor.c:245-276). */
static Tensor *dequantize(Tensor *in) {
    Tensor *out = tensor_create(in->dim, F32);
    out->vdim = in->vdim;
    out->hdim = in->hdim;
    for (size_t at = 0; at < in->dim; at += CONVERT_CHUNK) {
        const size_t n = in->dim - at < CONVERT_CHUNK ? in->dim - at : CONVERT_CHUNK;
        int8_t *q = dev_reserve(&g_q, CONVERT_CHUNK);
        float *s = dev_reserve(&g_s, CONVERT_CHUNK / 32 * sizeof(float));
        float *f = dev_reserve(&g_src, CONVERT_CHUNK * 4);
        host_check_cuda(cudaMemcpy(q, (const int8_t *)in->data + at, n, cudaMemcpyHostToDevice), "convert: copy values");
        host_check_cuda(cudaMemcpy(s, in->scale + at / 32, n / 32 * sizeof(float), cudaMemcpyHostToDevice),
                        "convert: copy scales");
        host_check(dk_dequantize_q8_0(q, s, n, f, NULL), "convert: dequantise");
        host_check_cuda(cudaMemcpy(data_f32(out) + at, f, n * sizeof(float), cudaMemcpyDeviceToHost),
                        "convert: copy back");
    }
    return out;
}

/* F16 / BF16 -> F32: exact widening (convert_f16_f32 / convert_bf16_f32, src/tensor.c:346-372). */
static Tensor *widen(Tensor *in) {
    Tensor *out = tensor_create(in->dim, F32);
    out->vdim = in->vdim;
    out->hdim = in->hdim;
    const uint16_t *src = (const uint16_t *)in->data;
    float *dst = data_f32(out);
    if (in->type == BF16)
        for (size_t i = 0; i < in->dim; ++i) dst[i] = bf16_to_float(src[i]);
    else
        for (size_t i = 0; i < in->dim; ++i) dst[i] = f16_to_float(src[i]);
    return out;
}

Tensor *convert(Tensor *input, quant_t type) {
    if (input->type == type) return input;  /* the reference returns the input itself */
    if (type == Q8_0 && (input->type == F32 || input->type == F16 || input->type == BF16)) return quantize(input);
    if (type == F32 && (input->type == F16 || input->type == BF16)) return widen(input);
    if (type == F32 && input->type == Q8_0) return dequantize(input);
    return NULL;
}
