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
    const uint8_t *w = nullptr;  // packed rows (q8_row_bytes(n) each)
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
    int RS = 0;        // packed row bytes
    int grid = 1;      // CTAs (one contiguous row range each)
    int CW = 4;        // consumer warps
    int SPW = 1;       // stage slots per consumer warp (warp w owns slots w*SPW .. w*SPW+SPW-1)
    size_t stage = 0;  // bytes of one stage (R packed rows)
    size_t ring = 0;   // bytes of all stages
    size_t xoff = 0;   // shared-memory offset of the activation
    size_t smem = 0;   // dynamic shared memory bytes
};

// ---- packed Q8_0 weight layout --------------------------------------------------------------
// A packed row is a sequence of 512-column blocks, padded to a multiple of 128 bytes.  Block b
// holds w_b = min(512, n - 512b) int8 values (w_b/16 chunks of 16 bytes) followed by their w_b/32
// fp32 scales, padded to 16 bytes; a full block is 576 bytes.  Inside a block the 16-byte chunks
// are XOR-swizzled by a row/segment key so that the GEMV's lanes read shared memory without bank
// conflicts (q8_swz_q / q8_swz_s).
//
// GEMV geometry of an n-column matrix: L lanes cooperate on one row (lane j handles the BL
// consecutive blocks starting at j*BL), R = 32/L rows per warp-stage.
struct Q8Geom {
    int nblk, L, BL, R;
};
__host__ __device__ inline size_t q8_row_bytes(int n);
// L is the smallest power of two (>= 8 when the row has more than 2 blocks, so an 8-lane shared
// memory phase stays inside one row) with at most 2 blocks per lane and a stage of R = 32/L rows
// of at most 25 KB.
__host__ __device__ inline Q8Geom q8_geom(int n) {
    Q8Geom g;
    g.nblk = (n + 511) / 512;
    const size_t rs = q8_row_bytes(n);
    g.L = g.nblk > 2 ? 8 : 1;
    while (g.L < 32 && ((g.nblk + g.L - 1) / g.L > 2 || (size_t)(32 / g.L) * rs > 25 * 1024)) g.L *= 2;
    g.BL = (g.nblk + g.L - 1) / g.L;
    g.R = 32 / g.L;
    return g;
}
__host__ __device__ inline int q8_blk_width(int n, int b) { return (n - 512 * b) < 512 ? (n - 512 * b) : 512; }
__host__ __device__ inline size_t q8_blk_bytes(int w) { return ((size_t)w + (size_t)w / 8 + 15) & ~(size_t)15; }
__host__ __device__ inline size_t q8_blk_off(int b) { return (size_t)b * 576; }
// Bytes of one packed row of an n-column matrix.
__host__ __device__ inline size_t q8_row_bytes(int n) {
    const size_t raw = (size_t)(n / 512) * 576 + ((n % 512) ? q8_blk_bytes(n % 512) : 0);
    return (raw + 127) & ~(size_t)127;
}
// Swizzle key of (packed row, block).
__host__ __device__ inline int q8_swz_key(const Q8Geom &g, int row, int b) { return (row * g.L + b / g.BL) & 7; }
// Physical position of value chunk c / scale chunk s of a block of width wb.
__host__ __device__ inline int q8_swz_q(int c, int key, int wb) { return ((wb / 16) % 8 == 0) ? (c ^ key) : c; }
__host__ __device__ inline int q8_swz_s(int s, int key, int wb) {
    const int nsc = wb / 128;  // scale chunks of a width that is a multiple of 128
    return (wb % 128 == 0 && (nsc == 1 || nsc == 2 || nsc == 4)) ? (s ^ (key & (nsc - 1))) : s;
}
// Element i of packed row `row` (dequantised): q * scale.
__host__ __device__ inline float q8_packed_elem(const uint8_t *rowp, int n, int row, int i) {
    const Q8Geom g = q8_geom(n);
    const int b = i >> 9, wb = q8_blk_width(n, b), key = q8_swz_key(g, row, b);
    const uint8_t *seg = rowp + q8_blk_off(b);
    const int within = i & 511;
    const int8_t q = (int8_t)seg[q8_swz_q(within >> 4, key, wb) * 16 + (within & 15)];
    const int grp = within >> 5;
    const float s = *reinterpret_cast<const float *>(seg + wb + q8_swz_s(grp >> 2, key, wb) * 16 + (grp & 3) * 4);
#ifdef __CUDA_ARCH__
    return __fmul_rn((float)q, s);
#else
    return (float)q * s;
#endif
}
// The 32 dequantised values of group g of packed row `row` (its two 16-byte chunks and one scale).
__host__ __device__ inline void q8_packed_group(const uint8_t *rowp, int n, int row, int g, float *f) {
    const Q8Geom gm = q8_geom(n);
    const int b = g >> 4, wb = q8_blk_width(n, b), key = q8_swz_key(gm, row, b), w = g & 15;
    const uint8_t *seg = rowp + q8_blk_off(b);
    const int8_t *c0 = reinterpret_cast<const int8_t *>(seg + 16 * q8_swz_q(2 * w, key, wb));
    const int8_t *c1 = reinterpret_cast<const int8_t *>(seg + 16 * q8_swz_q(2 * w + 1, key, wb));
    const float s = *reinterpret_cast<const float *>(seg + wb + 16 * q8_swz_s(w >> 2, key, wb) + 4 * (w & 3));
    for (int k = 0; k < 16; ++k) {
#ifdef __CUDA_ARCH__
        f[k] = __fmul_rn((float)c0[k], s);
        f[16 + k] = __fmul_rn((float)c1[k], s);
#else
        f[k] = (float)c0[k] * s;
        f[16 + k] = (float)c1[k] * s;
#endif
    }
}
size_t gemv_x_bytes(int n);
// ctas_per_sm: CTAs per SM (1 or 2); smem_budget: shared memory per SM for the stage rings
// (0 = default).  The ring of each CTA gets as many stage slots as fit, 1-3 per consumer warp.
GemvPlan plan_gemv(int n, int d, int epi, int num_sms, int ctas_per_sm = 1, size_t smem_budget = 0);
// Whether plan_gemv can serve this shape/epilogue (SwiGLU needs an even number of rows per stage).
bool gemv_supported(int n, int d, int epi);
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
