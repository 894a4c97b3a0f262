// gemv.cu -- the batch-1 Q8_0 GEMV (reference matmul_Q8_0, src/utils.c:106-138) for sm_100a.
//
// Weights live in HBM as packed rows: row r = n int8 values, then its n/32 fp32 scales, zero
// padding to 16 bytes (q8_row_bytes).  A CTA owns a contiguous range of row-blocks, so the bytes it
// streams are one contiguous range of HBM.
//
// Persistent kernel, one CTA per SM (two fit, so the next kernel's CTA can prefetch while this one
// drains).  Warp S (the last) is the producer: lane 0 streams row-blocks (R packed rows each) into a
// ring of S shared-memory stages with the bulk-copy engine (cp.async.bulk + mbarrier complete_tx,
// L2 evict-first).  The first S stages are issued BEFORE griddepcontrol.wait, i.e. while the
// previous kernel in the stream is still finishing, since weights do not depend on it.  Warps
// 0..S-1 are consumers; consumer w owns stage w.
//
// Numerics (bit-exact with the reference build): the activation is quantised with the reference's
// recipe (scale = amax*(1/127), q = rint(x*(1/scale))); per group the int32 dot is exact (dp4a);
// per row the fp32 sum is accumulated in group order as sum = sum + (float)dot * (w_scale*x_scale),
// no FMA -- the order and rounding of the reference's compiled loop.  Lanes compute 16 group
// products of a 512-byte slice in parallel; the ordered additions are then replayed on every lane
// from warp shuffles.
#include "dk_common.cuh"
#include "dk_kernels.h"

#include <algorithm>
#include <cmath>

namespace dk {

namespace {

constexpr int kMaxStages = 8;
constexpr int kMaxThreads = 32 * (kMaxStages + 1);

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (v != v) u = 0u;  // NaN never wins (the reference's strict '>' never selects it)
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}
__device__ __forceinline__ int argmax_idx(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
}

// Reference-order dot of one packed row (in shared memory) with the Q8_0 activation.
__device__ __forceinline__ float row_dot(const uint8_t *row, const int8_t *xq, const float *xs, int n,
                                         int lane) {
    const int C = n >> 4;  // 16-byte chunks; chunks 2g, 2g+1 form group g
    const float *ws = reinterpret_cast<const float *>(row + n);
    float sum = 0.0f;
    for (int base = 0; base < C; base += 32) {
        const int c = base + lane;
        int dot = 0;
        if (c < C) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(row + 16 * c);
            const uint4 xv = *reinterpret_cast<const uint4 *>(xq + 16 * c);
            dot = dp4a_16B(wv, xv);
        }
        dot += __shfl_xor_sync(FULL, dot, 1);
        float p = 0.0f;
        if (c < C) {
            const int g = c >> 1;
            p = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws[g], xs[g]));
        }
        const int ng = min(16, (C - base) >> 1);
        #pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float v = __shfl_sync(FULL, p, 2 * j);
            if (j < ng) sum = __fadd_rn(sum, v);
        }
    }
    return sum;
}

// Build the Q8_0 activation in shared memory (all threads of the CTA take part).
template <int PRO>
__device__ __forceinline__ void build_activation(const GemvArgs &a, int8_t *xq, float *xs, float *red) {
    const int tid = threadIdx.x, nthreads = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
    const int n = a.n, ng = n >> 5;
    if constexpr (PRO == PRO_Q8) {
        for (int i = tid; i < n / 16; i += nthreads)
            reinterpret_cast<uint4 *>(xq)[i] = reinterpret_cast<const uint4 *>(a.xq)[i];
        for (int i = tid; i < ng; i += nthreads) xs[i] = a.xs[i];
        return;
    } else {
        const int8_t *eq = nullptr;
        const float *es = nullptr;
        if constexpr (PRO == PRO_EMB_RMS) {
            // embedding row dequant (src/transformer.c:69 -> src/tensor.c:258-263)
            const int tok = a.tokens[*a.pos];
            const uint8_t *row = a.emb + (size_t)tok * q8_row_bytes(n);
            eq = reinterpret_cast<const int8_t *>(row);
            es = reinterpret_cast<const float *>(row + n);
        }
        auto load_x = [&](int i) -> float {
            if constexpr (PRO == PRO_EMB_RMS) return __fmul_rn((float)eq[i], es[i >> 5]);
            else return a.x[i];
        };
        float r = 1.0f;
        if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS) {
            float ss = 0.0f;
            for (int i = tid; i < n; i += nthreads) {
                const float v = load_x(i);
                if constexpr (PRO == PRO_EMB_RMS) {
                    if (blockIdx.x == 0) const_cast<float *>(a.x)[i] = v;  // residual stream x
                }
                ss = fmaf(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            if (warp == 0) {
                float t = lane < nwarps ? red[lane] : 0.0f;
                t = warp_sum(t);
                if (lane == 0) red[32] = t;
            }
            __syncthreads();
            // rmsnorm scale (src/utils.c:68-71): ss/n + 1e-5, then 1/sqrt.
            float v = __fdiv_rn(red[32], (float)n);
            v = __fadd_rn(v, 1e-5f);
            r = __fdiv_rn(1.0f, __fsqrt_rn(v));
        }
        for (int g = warp; g < ng; g += nwarps) {
            float v = load_x(32 * g + lane);
            if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS) v = __fmul_rn(__fmul_rn(a.norm_w[32 * g + lane], v), r);
            const float amax = warp_max(fabsf(v));
            float sc, inv;
            q8_scale(amax, sc, inv);
            xq[32 * g + lane] = (int8_t)q8_round(v, inv);
            if (lane == 0) xs[g] = sc;
        }
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kMaxThreads, 2) gemv_q8_kernel(const GemvArgs a, const GemvPlan p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = p.S, R = p.R, RS = p.RS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    uint8_t *ring = smem;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + p.ring);
    float *xs = reinterpret_cast<float *>(smem + p.ring + a.n);
    float *red = xs + (a.n >> 5);  // 40 floats
    uint64_t *full = reinterpret_cast<uint64_t *>(
        (reinterpret_cast<uintptr_t>(red + 40) + 7) & ~static_cast<uintptr_t>(7));
    uint64_t *empty = full + S;
    int *issued = reinterpret_cast<int *>(empty + S);  // per stage: copies issued
    int *consumed = issued + S;                         // per stage: copies waited for
    int *abort_flag = consumed + S;
    unsigned long long *wkey = reinterpret_cast<unsigned long long *>(
        (reinterpret_cast<uintptr_t>(abort_flag + 1) + 7) & ~static_cast<uintptr_t>(7));

    const int nblk = (a.d + R - 1) / R;
    const int b0 = (int)((long long)blockIdx.x * nblk / gridDim.x);
    const int b1 = (int)((long long)(blockIdx.x + 1) * nblk / gridDim.x);
    const int nb = b1 - b0;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            issued[s] = 0;
            consumed[s] = 0;
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    const bool producer = (warp == S) && (lane == 0);
    uint64_t policy = 0;
    auto issue = [&](int k) {
        const int row0 = (b0 + k) * R;
        const int rows = min(R, a.d - row0);
        const uint32_t bytes = (uint32_t)rows * (uint32_t)RS;
        const int slot = k % S;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * p.stage, a.w + (size_t)row0 * RS, bytes, &full[slot], policy);
        issued[slot] += 1;
    };
    if (producer) {
        policy = l2_evict_first_policy();
        const int first = min(S, nb);
        for (int k = 0; k < first; ++k) issue(k);  // weights only: safe before the dependency wait
    }

    pdl_wait();
    pdl_trigger();
    build_activation<PRO>(a, xq, xs, red);
    __syncthreads();

    unsigned long long best = 0ull;
    if (warp == S) {
        if (producer) {
            for (int k = S; k < nb; ++k) {
                const int slot = k % S;
                if (*reinterpret_cast<volatile int *>(abort_flag)) break;
                if (!mbar_wait(&empty[slot], (uint32_t)(((k / S) - 1) & 1), a.err)) {
                    *reinterpret_cast<volatile int *>(abort_flag) = 1;
                    break;
                }
                issue(k);
            }
        }
    } else {
        for (int k = warp; k < nb; k += S) {
            if (!mbar_wait(&full[warp], (uint32_t)((k / S) & 1), a.err)) {
                if (lane == 0) *reinterpret_cast<volatile int *>(abort_flag) = 1;
                break;
            }
            if (lane == 0) consumed[warp] += 1;
            const int row0 = (b0 + k) * R;
            const int rows = min(R, a.d - row0);
            const uint8_t *st = ring + (size_t)warp * p.stage;
            if constexpr (EPI == EPI_SWIGLU) {
                for (int r = 0; r + 1 < rows; r += 2) {
                    const float h1 = row_dot(st + (size_t)r * RS, xq, xs, a.n, lane);
                    const float h3 = row_dot(st + (size_t)(r + 1) * RS, xq, xs, a.n, lane);
                    if (lane == 0) {
                        // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                        float v = __fmul_rn(h1, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-h1))));
                        v = __fmul_rn(v, h3);
                        a.out[(row0 + r) >> 1] = v;
                    }
                }
            } else {
                for (int r = 0; r < rows; ++r) {
                    const float v = row_dot(st + (size_t)r * RS, xq, xs, a.n, lane);
                    const int row = row0 + r;
                    if (lane == 0) {
                        if constexpr (EPI == EPI_ADD) a.out[row] = __fadd_rn(a.out[row], v);
                        else a.out[row] = v;
                    }
                    if constexpr (EPI == EPI_ARGMAX) {
                        const unsigned long long key = argmax_key(v, row);
                        best = key > best ? key : best;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[warp]);
        }
        if constexpr (EPI == EPI_ARGMAX) {
            if (lane == 0) wkey[warp] = best;
        }
    }
    __syncthreads();

    // Error path only: never leave a bulk copy in flight into shared memory of an exiting CTA.
    if (tid == 0 && *reinterpret_cast<volatile int *>(abort_flag)) {
        for (int s = 0; s < S; ++s) {
            while (consumed[s] < issued[s]) {
                if (!mbar_wait(&full[s], (uint32_t)(consumed[s] & 1), a.err)) break;
                consumed[s] += 1;
            }
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        __shared__ int is_last;
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < S; ++w) b = wkey[w] > b ? wkey[w] : b;
            a.amax_part[blockIdx.x] = b;
            __threadfence();
            const unsigned ticket = atomicAdd(a.amax_count, 1u);
            is_last = (ticket == gridDim.x - 1);
        }
        __syncthreads();
        if (is_last && tid == 0) {
            __threadfence();
            unsigned long long b = 0ull;
            for (int i = 0; i < (int)gridDim.x; ++i) {
                const unsigned long long k = __ldcg(a.amax_part + i);
                b = k > b ? k : b;
            }
            int idx = (b == 0ull) ? 0 : argmax_idx(b);
            if (idx < 0 || idx >= a.d) idx = 0;
            const int pos = *a.pos;
            if (pos + 1 <= a.seq_len && pos + 1 >= *a.n_forced) a.tokens[pos + 1] = idx;
            *a.pos = pos + 1;
            *a.amax_count = 0u;
        }
    }
}

template <int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    auto kern = gemv_q8_kernel<PRO, EPI>;
    // Opt in to up to 227 KB of dynamic shared memory, once per device and template instance.
    static unsigned long long attr_done = 0ull;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!((attr_done >> dev) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_done |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(32 * (p.S + 1));
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, p);
}

}  // namespace

GemvPlan plan_gemv(int n, int d, int epi, int num_sms, size_t smem_budget) {
    GemvPlan p;
    p.RS = (int)q8_row_bytes(n);
    const int stage_target = 10 * 1024;
    int R = std::max(1, std::min(stage_target / p.RS, d / std::max(1, 2 * num_sms)));
    if (epi == EPI_SWIGLU) R = std::max(2, R & ~1);
    p.R = R;
    p.stage = ((size_t)R * p.RS + 127) & ~(size_t)127;
    // activation + reduction scratch + barriers/bookkeeping
    const size_t act = (size_t)n + (size_t)(n / 32) * 4 + 40 * 4 + 16 + kMaxStages * 16 + kMaxStages * 8 + 16 +
                       kMaxStages * 8 + 64;
    size_t budget = smem_budget ? smem_budget : 110 * 1024;  // two CTAs per SM
    int S = kMaxStages;
    while (S > 2 && S * p.stage + act > budget) --S;
    if (S < 4 && !smem_budget) {  // very long rows: one CTA per SM, deeper ring
        budget = 220 * 1024;
        S = kMaxStages;
        while (S > 2 && S * p.stage + act > budget) --S;
    }
    p.S = S;
    p.ring = (size_t)S * p.stage;
    p.smem = p.ring + act;
    const int nblk = (d + R - 1) / R;
    p.grid = std::max(1, std::min(num_sms, nblk));
    return p;
}

cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
#define DK_GEMV_CASE(P, E) \
    if (a.pro == P && a.epi == E) return launch_t<P, E>(a, p, st, pdl);
    DK_GEMV_CASE(PRO_Q8, EPI_STORE)
    DK_GEMV_CASE(PRO_F32, EPI_STORE)
    DK_GEMV_CASE(PRO_F32, EPI_ADD)
    DK_GEMV_CASE(PRO_RMS, EPI_STORE)
    DK_GEMV_CASE(PRO_RMS, EPI_SWIGLU)
    DK_GEMV_CASE(PRO_RMS, EPI_ARGMAX)
    DK_GEMV_CASE(PRO_EMB_RMS, EPI_STORE)
    DK_GEMV_CASE(PRO_F32, EPI_NONE)
#undef DK_GEMV_CASE
    return cudaErrorInvalidValue;
}

}  // namespace dk
