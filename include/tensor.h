/*
 * tensor.h -- the reference's Tensor container (src/tensor.h), served by libdiolkos.so.
 *
 * A Tensor is a HOST array: F32, F16 or BF16 values, or Q8_0 (int8 values followed by one fp32 scale
 * per 32 values, the reference's planar layout and cache-file layout).  Format conversions that do
 * arithmetic (quantisation, dequantisation) run on the current CUDA device through the C ABI in
 * diolkos.h; the decode path itself never uses host tensors (see transformer.h).
 */
#ifndef DIOLKOS_TENSOR_H
#define DIOLKOS_TENSOR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum quant_t { F32, F16, BF16, Q8_0, Q4_0 } quant_t;

/* Opaque element storage: a typed pointer so that tensor data is never converted implicitly. */
typedef struct TensorData TensorData;

typedef struct Tensor {
    quant_t type;
    TensorData *data;   /* dim elements of `type` (int8 for Q8_0)                         */
    float *scale;       /* Q8_0 only: dim/32 scales (stored right after the values)       */
    size_t dim;         /* element count                                                  */
    size_t hdim;        /* input dimension (columns) of a matrix                          */
    size_t vdim;        /* output dimension (rows) of a matrix                            */
    uint32_t tensor_id; /* kept for source compatibility (the reference's worker ids)     */
    int fd;             /* kept for source compatibility                                  */
} Tensor;

/* bf16 / IEEE half bit patterns to float (exact). */
float bf16_to_float(uint16_t bf16);
float f16_to_float(uint16_t f16);

/* A zero-filled host tensor of `size` elements (Q8_0: size % 32 == 0, scales allocated with it). */
Tensor *tensor_create(size_t size, quant_t type);
void tensor_destroy(Tensor *tensor);
/* Bytes of the tensor's element storage (values + scales for Q8_0). */
size_t Tensor_storage_size(Tensor *tensor);
size_t tensor_memory(Tensor *tensor);

/* A new tensor holding `input` converted to `type`: F32/F16/BF16 -> F32 or Q8_0, Q8_0 -> F32, or a copy
 * when the types match.  Quantisation follows the reference bit for bit (convert_bf16_q8_0 for bf16
 * weights, src/tensor.c:312-344; convert_f32_q8_slice_into_offset for fp32, :199-228) and runs on
 * the GPU.  NULL for an unsupported pair. */
Tensor *convert(Tensor *input, quant_t type);

float *data_f32(Tensor *tensor);
int8_t *data_i8(Tensor *tensor);

int group_size(quant_t type);          /* 32 for Q8_0 / Q4_0, 1 otherwise */
int quant_size(quant_t type);          /* bytes per stored element (1 for Q8_0) */
const char *quant_t_to_string(quant_t type);

#ifdef __cplusplus
}
#endif
#endif
