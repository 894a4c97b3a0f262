// attention.cu -- RoPE + KV-cache write + multi-head attention over the KV cache for one decode
// step (reference forward, src/transformer.c:87-193), as split-K flash-decoding on sm_100a.
//
// Grid (n_kv_heads, max_splits); CTA (kvh, s) serves every query head that shares KV head kvh
// (GQA: n_heads/n_kv_heads of them) over its slice of positions [t0, t1) of 0..pos.  The number
// of live splits is chosen on the device from pos (pos lives in device memory so that one captured
// CUDA graph serves every position); CTAs past it exit at once.
//
//  * RoPE (src/transformer.c:87-119, HF rotate-half): pairs (j, j+hs/2) rotated with the
//    precomputed (cos, sin) of this position, as the reference's compiled code evaluates it:
//    a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c).
//  * KV write (src/transformer.c:145-146): the CTA whose slice holds `pos` rotates k, rounds k and v
//    to the cache type (bf16 = upper 16 bits of the fp32 pattern, i.e. truncation; or fp32) and
//    stores them; the step then reads them back from the cache like the reference does.
//  * scores q.k / sqrtf(hs), softmax (expf), and sum_t a_t v_t (src/transformer.c:149-193): each
//    split keeps (max, sum, unnormalised accumulator); the last CTA of a KV head to finish merges
//    the splits and writes the heads' outputs.
//
// Cache layout per layer: [n_kv_heads][seq_len][head_size], so a head's positions are contiguous.
#include "dk_common.cuh"
#include "dk_kernels.h"

#include <algorithm>

namespace dk {
namespace {

constexpr int kAttnThreads = 128;  // head_size <= 128

template <bool F32>
struct KV;
template <>
struct KV<false> {
    using T = uint16_t;
    __device__ static float load(const T *p) { return __uint_as_float((uint32_t)(*p) << 16); }
    __device__ static T from_f32(float f) { return (T)(__float_as_uint(f) >> 16); }  // truncation
};
template <>
struct KV<true> {
    using T = float;
    __device__ static float load(const T *p) { return *p; }
    __device__ static T from_f32(float f) { return f; }
};

struct AttnGeom {
    int nsplit, chunk, t0, t1;
};

__device__ __forceinline__ AttnGeom attn_geom(int T, int split, int max_splits, int min_chunk) {
    AttnGeom g;
    g.nsplit = min(max_splits, (T + min_chunk - 1) / min_chunk);
    g.chunk = (T + g.nsplit - 1) / g.nsplit;
    g.t0 = split * g.chunk;
    g.t1 = min(T, g.t0 + g.chunk);
    return g;
}

template <bool F32>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
    using K = KV<F32>;
    using T = typename K::T;
    extern __shared__ __align__(16) float sm[];

    pdl_wait();
    pdl_trigger();

    const int kvh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int hs = a.head_size, half = hs >> 1;
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const int dim = a.n_heads * hs, kv_dim = a.n_kv_heads * hs;
    const int pos = *a.pos;
    if (pos < 0 || pos >= a.seq_len) {
        if (tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(a.err, DK_ERR_INVALID);
        return;
    }
    const int Tn = pos + 1;
    const AttnGeom g = attn_geom(Tn, split, a.max_splits, a.min_chunk);
    if (split >= g.nsplit) return;
    const int len = g.t1 - g.t0;
    const int chunk_max = (int)((a.seq_len + a.max_splits - 1) / a.max_splits) > a.min_chunk
                              ? (a.seq_len + a.max_splits - 1) / a.max_splits
                              : a.min_chunk;

    float *qs = sm;                        // [kv_mul][hs], rotated queries
    float *sc = qs + kv_mul * hs;          // [kv_mul][chunk_max], scores then exp
    float *stat = sc + kv_mul * chunk_max; // [kv_mul][2]: max, sum
    const float *rope = a.rope + (size_t)pos * hs;  // (cos, sin) pairs for j < hs/2

    // --- RoPE on the queries of this KV head's group
    for (int idx = tid; idx < kv_mul * half; idx += blockDim.x) {
        const int m = idx / half, j = idx - m * half;
        const float *q = a.qkv + (size_t)(kvh * kv_mul + m) * hs;
        const float c = rope[2 * j], s = rope[2 * j + 1];
        const float q0 = q[j], q1 = q[j + half];
        qs[m * hs + j] = __fmaf_rn(q0, c, -__fmul_rn(q1, s));
        qs[m * hs + j + half] = __fmaf_rn(q0, s, __fmul_rn(q1, c));
    }

    T *kc = reinterpret_cast<T *>(a.k_cache) + (size_t)kvh * a.seq_len * hs;
    T *vc = reinterpret_cast<T *>(a.v_cache) + (size_t)kvh * a.seq_len * hs;

    // --- this position's k (rotated) and v into the cache
    if (pos >= g.t0 && pos < g.t1) {
        const float *k = a.qkv + dim + (size_t)kvh * hs;
        const float *v = a.qkv + dim + kv_dim + (size_t)kvh * hs;
        for (int j = tid; j < half; j += blockDim.x) {
            const float c = rope[2 * j], s = rope[2 * j + 1];
            const float k0 = k[j], k1 = k[j + half];
            kc[(size_t)pos * hs + j] = K::from_f32(__fmaf_rn(k0, c, -__fmul_rn(k1, s)));
            kc[(size_t)pos * hs + j + half] = K::from_f32(__fmaf_rn(k0, s, __fmul_rn(k1, c)));
        }
        for (int i = tid; i < hs; i += blockDim.x) vc[(size_t)pos * hs + i] = K::from_f32(v[i]);
    }
    __syncthreads();

    // --- scores: warp per position, lanes over the head dimension
    const float sq = __fsqrt_rn((float)hs);
    for (int t = g.t0 + warp; t < g.t1; t += nwarps) {
        const T *kr = kc + (size_t)t * hs;
        float kv[4];
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = lane + 32 * e;
            kv[e] = i < hs ? K::load(kr + i) : 0.0f;
        }
        for (int m = 0; m < kv_mul; ++m) {
            float d = 0.0f;
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = lane + 32 * e;
                if (i < hs) d = __fmaf_rn(qs[m * hs + i], kv[e], d);
            }
            d = warp_sum(d);
            if (lane == 0) sc[m * chunk_max + (t - g.t0)] = __fdiv_rn(d, sq);
        }
    }
    __syncthreads();

    // --- per head: local max, exp, local sum
    for (int m = warp; m < kv_mul; m += nwarps) {
        float mx = -INFINITY;
        for (int t = lane; t < len; t += 32) mx = fmaxf(mx, sc[m * chunk_max + t]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int t = lane; t < len; t += 32) {
            const float e = expf(sc[m * chunk_max + t] - mx);
            sc[m * chunk_max + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            stat[2 * m] = mx;
            stat[2 * m + 1] = l;
        }
    }
    __syncthreads();

    // --- weighted sum of values: thread per head-dimension element
    float acc[8];
    #pragma unroll
    for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
    const int i = tid;
    if (i < hs) {
        for (int t = 0; t < len; ++t) {
            const float v = K::load(vc + (size_t)(g.t0 + t) * hs + i);
            #pragma unroll
            for (int m = 0; m < 8; ++m)
                if (m < kv_mul) acc[m] = __fmaf_rn(sc[m * chunk_max + t], v, acc[m]);
        }
    }

    if (g.nsplit == 1) {
        if (i < hs)
            for (int m = 0; m < kv_mul; ++m)
                a.out[(size_t)(kvh * kv_mul + m) * hs + i] = __fdiv_rn(acc[m], stat[2 * m + 1]);
        return;
    }

    // --- split partials, then the last CTA of this KV head merges them
    const int W = hs + 2;
    for (int m = 0; m < kv_mul; ++m) {
        float *w = a.work + ((size_t)(kvh * kv_mul + m) * a.max_splits + split) * W;
        if (tid == 0) {
            w[0] = stat[2 * m];
            w[1] = stat[2 * m + 1];
        }
        if (i < hs) w[2 + i] = acc[m];
    }
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (tid == 0) {
        const unsigned ticket = atomicAdd(a.count + kvh, 1u);
        is_last = (ticket == (unsigned)g.nsplit - 1u);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int m = 0; m < kv_mul; ++m) {
        const float *wb = a.work + (size_t)(kvh * kv_mul + m) * a.max_splits * W;
        float M = -INFINITY;
        for (int s = 0; s < g.nsplit; ++s) M = fmaxf(M, __ldcg(wb + (size_t)s * W));
        float L = 0.0f, o = 0.0f;
        for (int s = 0; s < g.nsplit; ++s) {
            const float f = expf(__ldcg(wb + (size_t)s * W) - M);
            L = __fmaf_rn(__ldcg(wb + (size_t)s * W + 1), f, L);
            if (i < hs) o = __fmaf_rn(__ldcg(wb + (size_t)s * W + 2 + i), f, o);
        }
        if (i < hs) a.out[(size_t)(kvh * kv_mul + m) * hs + i] = __fdiv_rn(o, L);
    }
    if (tid == 0) a.count[kvh] = 0u;
}

}  // namespace

int attn_max_splits(int seq_len, int n_kv_heads, int num_sms) {
    const int min_chunk = 64;
    int s = (4 * num_sms + n_kv_heads - 1) / n_kv_heads;
    s = std::max(1, std::min(s, (seq_len + min_chunk - 1) / min_chunk));
    return s;
}

size_t attn_smem_bytes(const AttnArgs &a) {
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const int chunk_max = std::max(a.min_chunk, (a.seq_len + a.max_splits - 1) / a.max_splits);
    return sizeof(float) * ((size_t)kv_mul * a.head_size + (size_t)kv_mul * chunk_max + 2 * (size_t)kv_mul);
}

size_t attn_count_offset(int n_heads, int head_size, int max_splits) {
    return ((size_t)n_heads * max_splits * (head_size + 2) * sizeof(float) + 255) & ~(size_t)255;
}

size_t attn_work_bytes(int n_heads, int n_kv_heads, int head_size, int max_splits) {
    return attn_count_offset(n_heads, head_size, max_splits) + (((size_t)n_kv_heads * 4 + 255) & ~(size_t)255);
}

bool attn_supported(int n_heads, int n_kv_heads, int head_size) {
    return n_heads > 0 && n_kv_heads > 0 && head_size > 0 && head_size <= 128 && !(head_size & 1) &&
           n_heads % n_kv_heads == 0 && n_heads / n_kv_heads <= 8;
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (!attn_supported(a.n_heads, a.n_kv_heads, a.head_size)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv_heads, a.max_splits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(a);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cfg.dynamicSmemBytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(a.kv_f32 ? attention_kernel<true> : attention_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
        if (e != cudaSuccess) return e;
    }
    if (a.kv_f32) return cudaLaunchKernelEx(&cfg, attention_kernel<true>, a);
    return cudaLaunchKernelEx(&cfg, attention_kernel<false>, a);
}

}  // namespace dk
