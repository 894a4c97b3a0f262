// q8.cu -- Q8_0 conversions, packing and small helpers (sm_100a).
//
//  * quant_16bit: convert_bf16_q8_0 / convert_f16_q8_0 (reference src/tensor.c:312-344, :278-310),
//    the load-time weight quantisers.
//  * quant_f32:  convert_f32_q8_slice_into_offset (src/tensor.c:199-228), the activation quantiser.
//  * dequant:    convert_q8_f32_slice_into_offset (src/tensor.c:245-265).
//  * group_dots: the exact int32 per-group dots of matmul_Q8_0 (src/utils.c:122-127).
//  * pack_rows:  planar cache layout -> packed GEMV rows.
//  * rmsnorm:    rmsnorm (src/utils.c:59-76) as a standalone kernel.
//  * embed:      the embedding-row dequant that starts forward (src/transformer.c:69).
// All of these are HBM-bound byte work: one thread per 32-element group, 16-byte loads and stores.
#include <cuda_fp16.h>

#include "dk_common.cuh"
#include "dk_kernels.h"

namespace dk {
namespace {

constexpr int kThreads = 256;

inline int grid_for(size_t items, int per_block = kThreads) {
    size_t g = (items + per_block - 1) / per_block;
    if (g > 148 * 32) g = 148 * 32;  // grid-stride beyond 32 CTAs per SM
    return (int)(g ? g : 1);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ void store_group(int8_t *q, const int (&v)[32]) {
    uint4 lo, hi;
    uint32_t w[8];
    #pragma unroll
    for (int k = 0; k < 8; ++k)
        w[k] = (uint32_t)(uint8_t)v[4 * k] | ((uint32_t)(uint8_t)v[4 * k + 1] << 8) |
               ((uint32_t)(uint8_t)v[4 * k + 2] << 16) | ((uint32_t)(uint8_t)v[4 * k + 3] << 24);
    lo = make_uint4(w[0], w[1], w[2], w[3]);
    hi = make_uint4(w[4], w[5], w[6], w[7]);
    reinterpret_cast<uint4 *>(q)[0] = lo;
    reinterpret_cast<uint4 *>(q)[1] = hi;
}

// Thread per group: amax over 32 values, scale = amax*(1/127), inv = 1/scale, q = rint(x*inv).
__device__ __forceinline__ void quant_group(const float (&f)[32], int8_t *q, float *s) {
    float amax = 0.0f;
    #pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(f[j]));
    float sc, inv;
    q8_scale(amax, sc, inv);
    int v[32];
    #pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = q8_round(f[j], inv);
    store_group(q, v);
    *s = sc;
}

// 16-bit source words to float, exactly: bf16 is the upper half of an fp32; IEEE half through the
// hardware conversion (exact for every half value, subnormals included).
struct Bf16Word {
    __device__ float operator()(uint16_t b) const { return bf16_to_f32(b); }
};
struct F16Word {
    __device__ float operator()(uint16_t h) const { return __half2float(__ushort_as_half(h)); }
};

template <typename Word>
__global__ void quant_16bit_kernel(const uint16_t *__restrict__ x, size_t ng, int8_t *__restrict__ q,
                                   float *__restrict__ s) {
    const Word cvt;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ng; g += (size_t)gridDim.x * blockDim.x) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + g * 32);
        float f[32];
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 u = __ldcs(src + k);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
            #pragma unroll
            for (int j = 0; j < 4; ++j) {
                f[8 * k + 2 * j] = cvt((uint16_t)(w[j] & 0xFFFF));
                f[8 * k + 2 * j + 1] = cvt((uint16_t)(w[j] >> 16));
            }
        }
        quant_group(f, q + g * 32, s + g);
    }
}

__global__ void quant_f32_kernel(const float *__restrict__ x, size_t ng, int8_t *__restrict__ q,
                                 float *__restrict__ s) {
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ng; g += (size_t)gridDim.x * blockDim.x) {
        const float4 *src = reinterpret_cast<const float4 *>(x + g * 32);
        float f[32];
        #pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 u = src[k];
            f[4 * k] = u.x; f[4 * k + 1] = u.y; f[4 * k + 2] = u.z; f[4 * k + 3] = u.w;
        }
        quant_group(f, q + g * 32, s + g);
    }
}

__global__ void dequant_kernel(const int8_t *__restrict__ q, const float *__restrict__ s, size_t n,
                               float *__restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn((float)q[i], s[i >> 5]);
}

__global__ void group_dots_kernel(const int8_t *__restrict__ xq, const int8_t *__restrict__ wq, int n, int d,
                                  int32_t *__restrict__ dots) {
    const int ng = n >> 5;
    const size_t total = (size_t)d * ng;
    for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
        const size_t row = t / ng;
        const int g = (int)(t - row * ng);
        const uint4 *w = reinterpret_cast<const uint4 *>(wq + row * n + (size_t)g * 32);
        const uint4 *x = reinterpret_cast<const uint4 *>(xq + (size_t)g * 32);
        dots[t] = dp4a_16B(w[0], x[0]) + dp4a_16B(w[1], x[1]);
    }
}

// Planar source row i -> packed row (row0 + i*step) of a tile-layout matrix with tile height T: per
// 512-column block, the row's segment (int8 values then fp32 scales, 16-byte chunks placed by the
// swizzle of the row's index in its tile).  The destination is zeroed beforehand, so the pad bytes of
// each segment and the rows of a ragged last tile stay zero.
__global__ void pack_rows_kernel(uint8_t *__restrict__ dst, int n, int T, const int8_t *__restrict__ q,
                                 const float *__restrict__ s, int row0, int step, int src_n, int col0) {
    const int i = blockIdx.x;  // source row
    const int drow = row0 + i * step, r = drow % T;
    const int8_t *qrow = q + (size_t)i * src_n + col0;
    const float *srow = s + (size_t)i * (src_n / 32) + col0 / 32;
    const int nblk = (n + 511) / 512;
    for (int b = 0; b < nblk; ++b) {
        const int wb = q8_blk_width(n, b);
        uint8_t *seg = dst + q8_seg_off(n, T, drow, b);
        const uint4 *qs = reinterpret_cast<const uint4 *>(qrow + 512 * b);
        for (int c = threadIdx.x; c < wb / 16; c += blockDim.x)
            reinterpret_cast<uint4 *>(seg)[q8_swz_q(c, r, wb)] = qs[c];
        for (int g = threadIdx.x; g < wb / 32; g += blockDim.x)
            reinterpret_cast<float *>(seg + wb + 16 * q8_swz_s(g >> 2, r, wb))[g & 3] = srow[16 * b + g];
    }
}

// One CTA: ss by tree reduction, scale = 1/sqrt(ss/n + 1e-5), o = (w*x)*scale.
__global__ void rmsnorm_kernel(float *o, const float *x, const float *w, int n) {
    __shared__ float red[33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    float ss = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nwarps ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    float v = __fdiv_rn(red[32], (float)n);
    v = __fadd_rn(v, 1e-5f);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(v));
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(w[i], x[i]), r);
}

// Dequantised embedding row tokens[*pos] (src/transformer.c:69), one thread per 32-value group.
__global__ void embed_kernel(const uint8_t *__restrict__ emb, int dim, int T, const int *tokens, const int *pos,
                             float *__restrict__ x) {
    pdl_wait();
    const int tok = tokens[*pos];
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < dim / 32; g += gridDim.x * blockDim.x) {
        float f[32];
        q8_packed_group(emb, dim, T, tok, g, f);
        float4 *o = reinterpret_cast<float4 *>(x + 32 * g);
        #pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = make_float4(f[4 * k], f[4 * k + 1], f[4 * k + 2], f[4 * k + 3]);
    }
    pdl_trigger();
}

}  // namespace

cudaError_t launch_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s, cudaStream_t st) {
    const size_t ng = n / 32;
    if (!ng) return cudaSuccess;
    quant_16bit_kernel<Bf16Word><<<grid_for(ng), kThreads, 0, st>>>(x, ng, q, s);
    return cudaGetLastError();
}

cudaError_t launch_quant_f16(const uint16_t *x, size_t n, int8_t *q, float *s, cudaStream_t st) {
    const size_t ng = n / 32;
    if (!ng) return cudaSuccess;
    quant_16bit_kernel<F16Word><<<grid_for(ng), kThreads, 0, st>>>(x, ng, q, s);
    return cudaGetLastError();
}

cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *q, float *s, cudaStream_t st) {
    const size_t ng = n / 32;
    if (!ng) return cudaSuccess;
    quant_f32_kernel<<<grid_for(ng), kThreads, 0, st>>>(x, ng, q, s);
    return cudaGetLastError();
}

cudaError_t launch_dequant(const int8_t *q, const float *s, size_t n, float *out, cudaStream_t st) {
    if (!n) return cudaSuccess;
    dequant_kernel<<<grid_for(n), kThreads, 0, st>>>(q, s, n, out);
    return cudaGetLastError();
}

cudaError_t launch_group_dots(const int8_t *xq, const int8_t *wq, int n, int d, int32_t *dots, cudaStream_t st) {
    const size_t total = (size_t)d * (n / 32);
    if (!total) return cudaSuccess;
    group_dots_kernel<<<grid_for(total), kThreads, 0, st>>>(xq, wq, n, d, dots);
    return cudaGetLastError();
}

cudaError_t launch_pack_rows(uint8_t *dst, int n, int T, const int8_t *q, const float *s, int rows, int row0,
                             int step, cudaStream_t st, int src_n, int col0) {
    if (rows <= 0) return cudaSuccess;
    if (src_n == 0) src_n = n;
    if (n <= 0 || n % 32 || T < 1 || T > 32 || src_n % 32 || col0 % 32 || col0 < 0 || col0 + n > src_n)
        return cudaErrorInvalidValue;
    pack_rows_kernel<<<rows, 128, 0, st>>>(dst, n, T, q, s, row0, step, src_n, col0);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float *o, const float *x, const float *w, int n, cudaStream_t st) {
    rmsnorm_kernel<<<1, 1024, 0, st>>>(o, x, w, n);
    return cudaGetLastError();
}

cudaError_t launch_embed(const uint8_t *emb_packed, int dim, int T, const int *tokens, const int *pos, float *x,
                         cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((dim / 32 + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, embed_kernel, emb_packed, dim, T, tokens, pos, x);
}

}  // namespace dk
