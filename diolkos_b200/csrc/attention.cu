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

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kBatch = 8;  // positions a warp loads at once (K and V rows together)

// 4 consecutive cache elements as floats, and back (the cache type's rounding: bf16 keeps the upper
// 16 bits of the fp32 pattern, i.e. truncates, like the reference's store, src/tensor.c:162-178).
template <bool F32>
__device__ __forceinline__ float4 load_kv4(const void *base, size_t idx) {
    if constexpr (F32) {
        return __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx));
    } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + idx));
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xFFFF0000u));
    }
}
template <bool F32>
__device__ __forceinline__ void store_kv4(void *base, size_t idx, float4 v) {
    if constexpr (F32) {
        *reinterpret_cast<float4 *>(static_cast<float *>(base) + idx) = v;
    } else {
        const uint2 u = make_uint2((__float_as_uint(v.x) >> 16) | (__float_as_uint(v.y) & 0xFFFF0000u),
                                   (__float_as_uint(v.z) >> 16) | (__float_as_uint(v.w) & 0xFFFF0000u));
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(base) + idx) = u;
    }
}
template <bool F32>
__device__ __forceinline__ float round_kv(float f) {
    if constexpr (F32) return f;
    else return __uint_as_float(__float_as_uint(f) & 0xFFFF0000u);
}

struct AttnGeom {
    int nsplit, chunk, t0, t1;
};

__device__ __forceinline__ AttnGeom attn_geom(int T, int split, int max_splits, int min_chunk) {
    AttnGeom g;
    attn_split_plan(T, max_splits, min_chunk, g.nsplit, g.chunk);
    g.t0 = split * g.chunk;
    g.t1 = min(T, g.t0 + g.chunk);
    return g;
}

// RoPE (src/transformer.c:87-119, HF rotate-half) of dims d0..d0+3 of the head vector v: pairs
// (j, j+hs/2) rotated by the (cos, sin) of this position, as the reference's compiled code evaluates
// them: a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c).
__device__ __forceinline__ float4 rope4(const float *v, const float *cs, int d0, int half) {
    float r[4];
    #pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int d = d0 + e;
        if (d < half) {
            const float c = cs[2 * d], sn = cs[2 * d + 1];
            r[e] = __fmaf_rn(v[d], c, -__fmul_rn(v[d + half], sn));
        } else {
            const int j = d - half;
            const float c = cs[2 * j], sn = cs[2 * j + 1];
            r[e] = __fmaf_rn(v[j], sn, __fmul_rn(v[d], c));
        }
    }
    return make_float4(r[0], r[1], r[2], r[3]);
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
    return __fmaf_rn(a.w, b.w, __fmaf_rn(a.z, b.z, __fmaf_rn(a.y, b.y, __fmul_rn(a.x, b.x))));
}

// CTA (kvh, split) serves the kv_mul query heads of KV head kvh over positions [t0, t1) of 0..pos.
// Lane l owns head dims 4l..4l+3; warp w takes the batches of kBatch positions starting at
// t0 + kBatch*(w + kAttnWarps*i) and keeps an online softmax (running max, sum, weighted V) per head.
template <bool F32>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];  // [kAttnWarps][kv_mul][hs + 4]: per-warp (max, sum, acc)

    pdl_wait();
    pdl_trigger();

    const int kvh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hs = a.head_size, half = hs >> 1;
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const int dim = a.n_heads * hs, kv_dim = a.n_kv_heads * hs;
    const int pos = *a.pos;
    if (pos < 0 || pos >= a.seq_len) {
        if (tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(a.err, DK_ERR_INVALID);
        return;
    }
    const AttnGeom g = attn_geom(pos + 1, split, a.max_splits, a.min_chunk);
    if (split >= g.nsplit) return;

    const int d0 = 4 * lane;
    const bool act = d0 < hs;
    const float *cs = a.rope + (size_t)pos * hs;  // (cos, sin) pairs for j < hs/2
    const size_t head_base = (size_t)kvh * a.seq_len * hs + d0;

    float4 q[8];
    #pragma unroll
    for (int m = 0; m < 8; ++m)
        q[m] = (m < kv_mul && act) ? rope4(a.qkv + (size_t)(kvh * kv_mul + m) * hs, cs, d0, half) : make_float4(0, 0, 0, 0);

    // This position's k (rotated) and v, rounded to the cache type; the split that holds `pos` stores
    // them and uses the rounded values as the cache row, like the reference reads them back.
    float4 kp = make_float4(0, 0, 0, 0), vp = kp;
    if (pos >= g.t0 && pos < g.t1 && act) {
        const float4 kr = rope4(a.qkv + dim + (size_t)kvh * hs, cs, d0, half);
        const float4 vr = *reinterpret_cast<const float4 *>(a.qkv + dim + kv_dim + (size_t)kvh * hs + d0);
        kp = make_float4(round_kv<F32>(kr.x), round_kv<F32>(kr.y), round_kv<F32>(kr.z), round_kv<F32>(kr.w));
        vp = make_float4(round_kv<F32>(vr.x), round_kv<F32>(vr.y), round_kv<F32>(vr.z), round_kv<F32>(vr.w));
        if (warp == 0) {
            store_kv4<F32>(a.k_cache, head_base + (size_t)pos * hs, kr);
            store_kv4<F32>(a.v_cache, head_base + (size_t)pos * hs, vr);
        }
    }

    const float sq = __fsqrt_rn((float)hs);
    float mx[8], l[8];
    float4 acc[8];
    #pragma unroll
    for (int m = 0; m < 8; ++m) {
        mx[m] = -INFINITY;
        l[m] = 0.0f;
        acc[m] = make_float4(0, 0, 0, 0);
    }
    for (int tb = g.t0 + warp * kBatch; tb < g.t1; tb += kAttnWarps * kBatch) {
        float4 kk[kBatch], vv[kBatch];
        #pragma unroll
        for (int j = 0; j < kBatch; ++j) {  // all loads of the batch first: one memory round trip
            const int t = tb + j;
            if (t < g.t1 && act && t != pos) {
                kk[j] = load_kv4<F32>(a.k_cache, head_base + (size_t)t * hs);
                vv[j] = load_kv4<F32>(a.v_cache, head_base + (size_t)t * hs);
            } else {
                kk[j] = (t == pos) ? kp : make_float4(0, 0, 0, 0);
                vv[j] = (t == pos) ? vp : make_float4(0, 0, 0, 0);
            }
        }
        #pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m >= kv_mul) break;
            float sc[kBatch];
            float bmax = -INFINITY;
            #pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                // score = q.k / sqrtf(head_size) (src/transformer.c:158-163)
                const float d = warp_sum(dot4(q[m], kk[j]));
                sc[j] = (tb + j < g.t1) ? __fdiv_rn(d, sq) : -INFINITY;
                bmax = fmaxf(bmax, sc[j]);
            }
            const float mnew = fmaxf(mx[m], bmax);
            const float rescale = expf(mx[m] - mnew);
            float lm = __fmul_rn(l[m], rescale);
            float4 am = make_float4(__fmul_rn(acc[m].x, rescale), __fmul_rn(acc[m].y, rescale),
                                    __fmul_rn(acc[m].z, rescale), __fmul_rn(acc[m].w, rescale));
            #pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const float pj = expf(sc[j] - mnew);
                lm = __fadd_rn(lm, pj);
                am.x = __fmaf_rn(pj, vv[j].x, am.x);
                am.y = __fmaf_rn(pj, vv[j].y, am.y);
                am.z = __fmaf_rn(pj, vv[j].z, am.z);
                am.w = __fmaf_rn(pj, vv[j].w, am.w);
            }
            mx[m] = mnew;
            l[m] = lm;
            acc[m] = am;
        }
    }

    // Merge the warps' partial softmaxes.  Shared layout per (warp, head): max, sum, 2 pad floats,
    // then the hs accumulators (16-byte aligned: hs % 4 == 0).
    const int W = hs + 2, SW = hs + 4;
    #pragma unroll
    for (int m = 0; m < 8; ++m) {
        if (m >= kv_mul) break;
        float *cw = sm + (size_t)(warp * kv_mul + m) * SW;
        if (lane == 0) {
            cw[0] = mx[m];
            cw[1] = l[m];
        }
        if (act) *reinterpret_cast<float4 *>(cw + 4 + d0) = acc[m];
    }
    __syncthreads();
    for (int m = 0; m < kv_mul; ++m) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm[(size_t)(w * kv_mul + m) * SW]);
        float L = 0.0f, o = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float *cw = sm + (size_t)(w * kv_mul + m) * SW;
            const float f = expf(cw[0] - M);  // 0 for a warp that had no positions (max = -inf)
            L = __fmaf_rn(cw[1], f, L);
            if (tid < hs) o = __fmaf_rn(cw[4 + tid], f, o);
        }
        if (g.nsplit == 1) {
            if (tid < hs) a.out[(size_t)(kvh * kv_mul + m) * hs + tid] = __fdiv_rn(o, L);
        } else {
            float *w = a.work + ((size_t)(kvh * kv_mul + m) * a.max_splits + split) * W;
            if (tid == 0) {
                w[0] = M;
                w[1] = L;
            }
            if (tid < hs) w[2 + tid] = o;
        }
    }
    if (g.nsplit == 1) return;

    // The last CTA of this KV head to finish merges the splits.
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
            if (tid < hs) o = __fmaf_rn(__ldcg(wb + (size_t)s * W + 2 + tid), f, o);
        }
        if (tid < hs) a.out[(size_t)(kvh * kv_mul + m) * hs + tid] = __fdiv_rn(o, L);
    }
    if (tid == 0) a.count[kvh] = 0u;
}

}  // namespace

int attn_max_splits(int seq_len, int n_kv_heads, int num_sms) {
    const int min_chunk = kAttnMinChunk;
    int s = (4 * num_sms + n_kv_heads - 1) / n_kv_heads;
    s = std::max(1, std::min(s, (seq_len + min_chunk - 1) / min_chunk));
    return s;
}

size_t attn_smem_bytes(const AttnArgs &a) {
    const int kv_mul = a.n_heads / a.n_kv_heads;
    return sizeof(float) * (size_t)kAttnWarps * kv_mul * (a.head_size + 4);
}

size_t attn_count_offset(int n_heads, int head_size, int max_splits) {
    return ((size_t)n_heads * max_splits * (head_size + 2) * sizeof(float) + 255) & ~(size_t)255;
}

size_t attn_work_bytes(int n_heads, int n_kv_heads, int head_size, int max_splits) {
    return attn_count_offset(n_heads, head_size, max_splits) + (((size_t)n_kv_heads * 4 + 255) & ~(size_t)255);
}

bool attn_supported(int n_heads, int n_kv_heads, int head_size) {
    return n_heads > 0 && n_kv_heads > 0 && head_size > 0 && head_size <= 128 && head_size % 4 == 0 &&
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
