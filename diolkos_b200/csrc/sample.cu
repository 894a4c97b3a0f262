// sample.cu -- token sampling and softmax on the GPU (reference sample(), src/sampler.c:108-131, and
// softmax_f32, src/utils.c:39-57).
//
// One CTA of 1024 threads over the n logits; thread t owns the contiguous values [t*C, (t+1)*C),
// C = ceil(n/1024), so index-ordered scans are a per-thread walk plus a block scan.
//
//  * temperature == 0: argmax, the first index winning ties (sample_argmax, src/sampler.c:6-17).
//  * temperature > 0: p = softmax(logits / temperature) (the reference divides each logit by the
//    temperature, then takes the softmax), then with the caller's coin in [0, 1):
//      - top-p off (topp <= 0 or >= 1): the first index whose cumulative probability, in index order,
//        exceeds the coin (sample_mult, src/sampler.c:19-30);
//      - top-p (src/sampler.c:40-83): the reference keeps the candidates p >= (1-topp)/(n-1), sorts
//        them by decreasing p, truncates after the first element where the running sum exceeds topp,
//        and walks that list to r = coin * (the truncated sum).  Here both cut points are found
//        without sorting: the truncation value v* is the largest u with sum(p >= u) > topp, and the
//        sampled value w the largest u with sum over the truncated set of (p >= u) > r -- two
//        bisections over the bit patterns of positive floats (their order is the value order).  The
//        token is the lowest index holding w.  Sums run in a different order than the reference's
//        sequential ones, so a coin landing within rounding of a boundary can pick the neighbour.
// Probabilities are recomputed from the logits on every pass (no scratch memory, any n).
#include "dk_common.cuh"
#include "dk_internal.h"

#include <cfloat>

namespace dk {
namespace {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ unsigned long long sample_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (v != v) u = 0u;  // NaN never wins
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}

// Block-wide reductions (1024 threads = 32 warps); `sh` holds 32 entries.
__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
    return t;
}
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = -FLT_MAX;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, sh[w]);
    return t;
}
__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *sh) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(FULL, v, o);
        v = w > v ? w : v;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long t = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = sh[w] > t ? sh[w] : t;
    return t;
}

struct Probs {  // p_i = expf(logits[i] / temperature - mx) / sum
    const float *logits;
    float temperature, mx, sum;
    __device__ float scaled(int i) const { return __fdiv_rn(logits[i], temperature); }
    __device__ float operator()(int i) const { return __fdiv_rn(expf(__fsub_rn(scaled(i), mx)), sum); }
};

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const float *logits, int n, float temperature,
                                                             float topp, float coin, float *probs, int *out) {
    __shared__ float shf[32];
    __shared__ unsigned long long shk[32];
    __shared__ float scan[kSampleThreads];
    __shared__ int s_pick;
    const int tid = threadIdx.x, C = (n + kSampleThreads - 1) / kSampleThreads;
    const int i0 = min(n, tid * C), i1 = min(n, i0 + C);

    if (temperature == 0.0f) {
        unsigned long long best = 0ull;
        for (int i = i0; i < i1; ++i) {
            const unsigned long long k = sample_key(logits[i], i);
            best = k > best ? k : best;
        }
        best = block_max_u64(best, shk);
        if (tid == 0) *out = best ? (int)(0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFull)) : 0;
        return;
    }

    if (tid == 0) s_pick = n - 1;
    Probs P{logits, temperature, 0.0f, 1.0f};
    float mx = -FLT_MAX;
    for (int i = i0; i < i1; ++i) mx = fmaxf(mx, P.scaled(i));
    P.mx = block_max(mx, shf);
    float s = 0.0f;
    for (int i = i0; i < i1; ++i) s = __fadd_rn(s, expf(__fsub_rn(P.scaled(i), P.mx)));
    P.sum = block_sum(s, shf);

    if (topp <= 0.0f || topp >= 1.0f) {
        // Cumulative probability in index order: chunk sums, then a block exclusive scan.
        float cs = 0.0f;
        for (int i = i0; i < i1; ++i) cs = __fadd_rn(cs, P(i));
        scan[tid] = cs;
        __syncthreads();
        if (tid == 0) {
            float run = 0.0f;
            for (int t = 0; t < kSampleThreads; ++t) {
                const float v = scan[t];
                scan[t] = run;
                run = __fadd_rn(run, v);
            }
        }
        __syncthreads();
        // Exactly one thread owns the coin: the one whose chunk starts at or below it and the next
        // chunk above it (the thread holding index n-1 also takes a coin beyond the total, which the
        // reference answers with n-1 as well).
        const int last = (n - 1) / C;
        const float base = scan[tid];
        if (tid <= last && !(coin < base) && (tid == last || coin < scan[tid + 1])) {
            float cdf = base;
            int pick = i1 - 1;
            for (int i = i0; i < i1; ++i) {
                cdf = __fadd_rn(cdf, P(i));
                if (coin < cdf) {
                    pick = i;
                    break;
                }
            }
            s_pick = pick;
        }
    } else {
        // Top-p.  mass(u) = sum of the candidates' p with p >= u; bisection for the largest u
        // (as a float bit pattern, 0 .. 1.0f) with mass(u) > limit.
        const float cutoff = __fdiv_rn(__fsub_rn(1.0f, topp), (float)(n - 1));
        auto mass = [&](float u, float floor_v) -> float {
            float m = 0.0f;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                if (p >= cutoff && p >= floor_v && p >= u) m = __fadd_rn(m, p);
            }
            return block_sum(m, shf);
        };
        auto largest = [&](float limit, float floor_v, bool &found) -> float {
            unsigned lo = 0u, hi = __float_as_uint(1.0f) + 1u;  // mass(lo) > limit ? ; mass(hi) == 0
            found = mass(__uint_as_float(lo), floor_v) > limit;
            if (!found) return 0.0f;
            while (hi - lo > 1u) {  // invariant: mass(lo) > limit, mass(hi) <= limit
                const unsigned mid = lo + (hi - lo) / 2u;
                if (mass(__uint_as_float(mid), floor_v) > limit) lo = mid;
                else hi = mid;
            }
            return __uint_as_float(lo);
        };
        bool found = false;
        // v*: the truncation value; without one (the candidates' sum does not exceed topp after
        // rounding) every candidate stays, as in the reference.
        const float vstar_raw = largest(topp, 0.0f, found);
        const float vstar = found ? vstar_raw : 0.0f;
        const float kept = mass(vstar, 0.0f);
        const float r = __fmul_rn(coin, kept);
        bool found_w = false;
        float w = largest(r, vstar, found_w);
        if (!found_w) {  // rounding: the reference returns the last kept element (the smallest p)
            float mn = FLT_MAX;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                if (p >= cutoff && p >= vstar) mn = fminf(mn, p);
            }
            w = -block_max(-mn, shf);
        }
        // The lowest index holding value w among the kept candidates.
        unsigned long long best = 0ull;
        for (int i = i0; i < i1; ++i) {
            const float p = P(i);
            if (p == w && p >= cutoff && p >= vstar) {
                const unsigned long long k = 0xFFFFFFFFull - (unsigned long long)i;
                best = k > best ? k : best;
            }
        }
        best = block_max_u64(best, shk);
        if (tid == 0 && best) s_pick = (int)(0xFFFFFFFFu - (unsigned)best);
    }
    // Every read of the logits is done before any probability is stored (probs may alias them).
    __syncthreads();
    if (probs)
        for (int i = i0; i < i1; ++i) probs[i] = P(i);
    if (tid == 0) *out = s_pick;
}

// softmax_f32 in place (one CTA): x = expf(x - max) / sum.
__global__ void __launch_bounds__(kSampleThreads) softmax_kernel(float *x, int n) {
    __shared__ float shf[32];
    const int tid = threadIdx.x, C = (n + kSampleThreads - 1) / kSampleThreads;
    const int i0 = min(n, tid * C), i1 = min(n, i0 + C);
    float mx = -FLT_MAX;
    for (int i = i0; i < i1; ++i) mx = fmaxf(mx, x[i]);
    mx = block_max(mx, shf);
    float s = 0.0f;
    for (int i = i0; i < i1; ++i) {
        const float e = expf(__fsub_rn(x[i], mx));
        x[i] = e;
        s = __fadd_rn(s, e);
    }
    s = block_sum(s, shf);
    for (int i = i0; i < i1; ++i) x[i] = __fdiv_rn(x[i], s);
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_sample(const float *logits, int n, float temperature, float topp, float coin, float *probs, int *out,
                         void *stream) {
    if (!logits || !out || n < 1) return set_error(DK_ERR_INVALID, "dk_sample: bad arguments");
    if (!(temperature >= 0.0f) || !(coin >= 0.0f && coin < 1.0f))
        return set_error(DK_ERR_INVALID, "dk_sample: temperature must be >= 0 and coin in [0, 1)");
    sample_kernel<<<1, kSampleThreads, 0, (cudaStream_t)stream>>>(logits, n, temperature, topp, coin, probs, out);
    return cuda_status(cudaGetLastError(), "dk_sample");
}

extern "C" int dk_softmax(float *x, int n, void *stream) {
    if (!x || n < 1) return set_error(DK_ERR_INVALID, "dk_softmax: bad arguments");
    softmax_kernel<<<1, kSampleThreads, 0, (cudaStream_t)stream>>>(x, n);
    return cuda_status(cudaGetLastError(), "dk_softmax");
}
