// dk_kernels.h -- host-side launch interface of the Diolkos B200 kernels (internal to the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dk {

// ---------------- GEMV -----------------------------------------------------------------------
// Activation prologue: how the CTA builds the Q8_0 activation in shared memory.
enum GemvPro : int {
    PRO_Q8 = 0,       // already quantised: xq int8[n], xs fp32[n/32]
    PRO_F32 = 1,      // quantise fp32 x[n] (convert_f32_q8, src/tensor.c:199)
    PRO_RMS = 2,      // rmsnorm(x, norm_w) then quantise (src/utils.c:59 + src/tensor.c:199)
    PRO_EMB_RMS = 3,  // x = dequant(embedding row tokens[*pos]) (written back by CTA 0), then as PRO_RMS
};
// Epilogue: what happens to each finished row value.
enum GemvEpi : int {
    EPI_STORE = 0,   // out[row] = v
    EPI_ADD = 1,     // out[row] += v (residual, src/transformer.c:199-201, :228-230)
    EPI_SWIGLU = 2,  // rows (2i, 2i+1) = (w1_i, w3_i): out[i] = silu(v0) * v1 (src/transformer.c:212-222)
    EPI_ARGMAX = 3,  // out[row] = v, and the greedy token (src/sampler.c:6-17) is written to tokens[pos+1]
    EPI_NONE = 4,    // partial sums only (tensor-parallel split: the caller reduces)
};

struct GemvArgs {
    const uint8_t *w = nullptr;  // packed rows (dk_q8_row_bytes(n) each)
    int n = 0, d = 0;
    int pro = PRO_F32, epi = EPI_STORE;
    const float *x = nullptr;       // PRO_F32 / PRO_RMS input; PRO_EMB_RMS: x is written here
    const float *norm_w = nullptr;  // PRO_RMS / PRO_EMB_RMS
    const int8_t *xq = nullptr;     // PRO_Q8
    const float *xs = nullptr;
    const uint8_t *emb = nullptr;   // PRO_EMB_RMS: packed embedding rows
    float *out = nullptr;
    // greedy-token epilogue and embedding prologue state (device memory)
    unsigned long long *amax_part = nullptr;  // >= grid entries
    unsigned int *amax_count = nullptr;       // zero between launches
    int *tokens = nullptr;                    // token buffer (capacity >= seq_len + 1)
    int *pos = nullptr;                       // current position (incremented by EPI_ARGMAX)
    const int *n_forced = nullptr;            // prompt length: tokens[0..n_forced) are forced
    int seq_len = 0;
    int *err = nullptr;                       // device error word
};

struct GemvPlan {
    int R = 1;        // rows per stage
    int S = 8;        // stages == consumer warps
    int RS = 0;       // packed row bytes
    int grid = 1;
    size_t smem = 0;  // dynamic shared memory bytes
    size_t ring = 0;  // bytes of the stage ring
    size_t stage = 0; // bytes of one stage
};

// Packed row bytes of an n-column Q8_0 matrix: n int8 + n/32 fp32 scales, padded to 16 bytes.
__host__ __device__ inline size_t q8_row_bytes(int n) { return ((size_t)n + (size_t)n / 8 + 15) & ~(size_t)15; }
GemvPlan plan_gemv(int n, int d, int epi, int num_sms, size_t smem_budget = 0);
cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl);

// ---------------- Q8_0 conversions ----------------------------------------------------------
cudaError_t launch_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s, cudaStream_t st);
cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *q, float *s, cudaStream_t st);
cudaError_t launch_dequant(const int8_t *q, const float *s, size_t n, float *out, cudaStream_t st);
cudaError_t launch_group_dots(const int8_t *xq, const int8_t *wq, int n, int d, int32_t *dots, cudaStream_t st);
cudaError_t launch_pack_rows(uint8_t *dst, int n, const int8_t *q, const float *s, int rows, int row0,
                             int step, cudaStream_t st);
cudaError_t launch_rmsnorm(float *o, const float *x, const float *w, int n, cudaStream_t st);
cudaError_t launch_embed(const uint8_t *emb_packed, int dim, const int *tokens, const int *pos, float *x,
                         cudaStream_t st, bool pdl);

// ---------------- attention ------------------------------------------------------------------
struct AttnArgs {
    const float *qkv = nullptr;  // [dim + 2*kv_dim]: q | k | v before RoPE
    const float *rope = nullptr; // [seq_len][head_size/2][2] (cos, sin)
    void *k_cache = nullptr;     // this layer: [n_kv_heads][seq_len][head_size], bf16 or f32
    void *v_cache = nullptr;
    float *out = nullptr;        // [n_heads*head_size]
    float *work = nullptr;       // split partials: [n_heads][max_splits][head_size + 2]
    unsigned int *count = nullptr; // [n_kv_heads] arrival counters (zero between launches)
    const int *pos = nullptr;
    int n_heads = 0, n_kv_heads = 0, head_size = 0, seq_len = 0;
    int kv_f32 = 0;
    int max_splits = 1, min_chunk = 64;
    int *err = nullptr;
};
int attn_max_splits(int seq_len, int n_kv_heads, int num_sms);
size_t attn_smem_bytes(const AttnArgs &a);
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl);

}  // namespace dk
