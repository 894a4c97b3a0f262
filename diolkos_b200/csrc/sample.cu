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
//        them by decreasing p (equal p stay in index order: glibc's qsort is a stable merge sort),
//        truncates after the first element where the running sum exceeds topp, and walks that list
//        to r = coin * (the truncated sum).  Here both cut points are found without sorting: the
//        truncation value v* is the largest u with sum(p >= u) > topp, the sampled value w the
//        largest u with sum over the kept list of (p >= u) > r -- bisections over the bit patterns
//        of positive floats (their order is the value order) -- and inside a group of equal
//        values the position follows from the group's start sum, so the token is the k-th index
//        holding that value.  Sums run in a different order than the reference's sequential ones,
//        so a coin landing within rounding of a boundary can pick the neighbour.
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
        // Top-p over the candidates p >= cutoff, in the reference's sorted order: decreasing p,
        // equal p in increasing index (the order its stable qsort leaves them in).  With
        // G(u) = sum of candidate p >= u, the running sum of that order passes through
        // G(>v) + j*v for the j-th of the c_v candidates equal to v.
        const float cutoff = __fdiv_rn(__fsub_rn(1.0f, topp), (float)(n - 1));
        auto mass = [&](float u) -> float {
            float m = 0.0f;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                if (p >= cutoff && p >= u) m = __fadd_rn(m, p);
            }
            return block_sum(m, shf);
        };
        auto count = [&](float v) -> int {
            float c = 0.0f;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                c += (p >= cutoff && p == v) ? 1.0f : 0.0f;
            }
            return (int)block_sum(c, shf);  // exact: counts stay far below 2^24
        };
        auto above = [](float v) { return __uint_as_float(__float_as_uint(v) + 1u); };
        // The largest u >= lo (positive floats compare like their bit patterns) with G(u) > limit:
        // always one of the candidate values.
        auto largest = [&](float lo_v, float limit, bool &found) -> float {
            unsigned lo = __float_as_uint(lo_v), hi = __float_as_uint(1.0f) + 1u;
            found = mass(lo_v) > limit;
            if (!found) return 0.0f;
            while (hi - lo > 1u) {  // invariant: G(lo) > limit, G(hi) <= limit
                const unsigned mid = lo + (hi - lo) / 2u;
                if (mass(__uint_as_float(mid)) > limit) lo = mid;
                else hi = mid;
            }
            return __uint_as_float(lo);
        };
        // Smallest j in [1, c] with g + j*v > limit (the first place the running sum passes it).
        auto first_past = [](float g, float v, int c, float limit) -> int {
            int j = (int)fminf(fmaxf(floorf(__fdiv_rn(__fsub_rn(limit, g), v)) + 1.0f, 1.0f), (float)c);
            while (j > 1 && __fadd_rn(g, __fmul_rn((float)(j - 1), v)) > limit) --j;
            while (j < c && !(__fadd_rn(g, __fmul_rn((float)j, v)) > limit)) ++j;
            return j;
        };
        // The truncation: the element where the running sum first exceeds topp is the j*-th
        // candidate equal to v*; the kept list ends there.  Without one (the candidates' sum does
        // not exceed topp after rounding) every candidate is kept.
        bool trunc = false;
        const float vstar = largest(0.0f, topp, trunc);
        float kept, last_v;
        int jstar = 0, last_k;
        if (trunc) {
            const float g_gt = mass(above(vstar));
            jstar = first_past(g_gt, vstar, count(vstar), topp);
            kept = __fadd_rn(g_gt, __fmul_rn((float)jstar, vstar));
            last_v = vstar;
            last_k = jstar - 1;
        } else {
            kept = mass(0.0f);
            float mn = FLT_MAX;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                if (p >= cutoff) mn = fminf(mn, p);
            }
            last_v = -block_max(-mn, shf);
            last_k = count(last_v) - 1;
        }
        // The sampled element: the first whose running sum exceeds r = coin * kept.
        const float r = __fmul_rn(coin, kept);
        bool hit = false;
        float w = largest(trunc ? above(vstar) : 0.0f, r, hit);
        if (!hit && trunc && r < kept) {  // r falls among the kept candidates equal to v*
            w = vstar;
            hit = true;
        }
        float pick_v = last_v;  // rounding: the reference returns the last kept element
        int pick_k = last_k;
        if (hit) {
            const float g_gt = mass(above(w));
            const int c = (trunc && w == vstar) ? jstar : count(w);
            pick_v = w;
            pick_k = first_past(g_gt, w, c, r) - 1;
        }
        // The pick_k-th (0-based, in index order) candidate equal to pick_v.
        int c = 0;
        for (int i = i0; i < i1; ++i) {
            const float p = P(i);
            c += (p >= cutoff && p == pick_v) ? 1 : 0;
        }
        __syncthreads();
        scan[tid] = (float)c;
        __syncthreads();
        if (tid == 0) {
            float run = 0.0f;
            for (int t = 0; t < kSampleThreads; ++t) {
                const float v = scan[t];
                scan[t] = run;
                run += v;
            }
        }
        __syncthreads();
        const int base = (int)scan[tid];
        if (pick_k >= base && pick_k < base + c) {
            int seen = base;
            for (int i = i0; i < i1; ++i) {
                const float p = P(i);
                if (p >= cutoff && p == pick_v) {
                    if (seen == pick_k) {
                        s_pick = i;
                        break;
                    }
                    ++seen;
                }
            }
        }
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
