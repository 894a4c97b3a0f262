// gemv.cu -- the batch-1 Q8_0 GEMV (reference matmul_Q8_0, src/utils.c:106-138) for sm_100a.
//
// Weights are packed rows (dk_kernels.h: 512-column blocks of int8 values + fp32 scales, chunks
// XOR-swizzled, rows padded to 128 bytes).  Persistent kernel, one CTA per SM: CTA c owns the
// contiguous rows [r0, r1), balanced to one row.  Its rows are streamed in stages of R = 32/L
// consecutive packed rows -- one contiguous range, ONE bulk copy (cp.async.bulk, 18-25 KB for the
// LLaMA shapes, L2 evict-first) completing on an mbarrier -- into a ring of stage slots filling the
// SM's shared memory (~150-200 KB in flight per SM: under full load a bulk copy takes ~2.5 us).
// Warp 4 is the producer; it issues the first ring-full of stages BEFORE griddepcontrol.wait, i.e.
// while the previous kernel in the stream is still running (weights never depend on it).  Consumer
// warp w takes stages w, w+4, w+8, ... into its own SPW slots; since each slot has one consumer that
// waits for its uses in order, the mbarrier phase parities never alias.
//
// Consumer warp, one stage: lane (r, j) = (lane / L, lane % L) takes row r of the stage and its
// blocks [j*BL, j*BL + BL).  Phase A: the lane computes, for each of its 32-element groups, the
// exact int32 dot (dp4a) and the product (float)dot * (w_scale * x_scale).  The stage is then handed
// back to the producer.  Phase B: the row's sum is accumulated in group order, sum = sum + product,
// no FMA -- the order and rounding of the reference's compiled loop -- the running sum hopping from
// lane (r, j) to lane (r, j+1) by shuffle.  The result is bit-identical to the reference build.
#include "dk_common.cuh"
#include "dk_kernels.h"

#include <algorithm>
#include <cmath>

namespace dk {
namespace {

constexpr int kThreads = 160;  // warps 0..3 consume, warp 4 produces; all build the activation
constexpr int kProducer = 4;
constexpr int kCW = 4;      // consumer warps
constexpr int kMaxSPW = 3;  // stage slots per consumer warp
constexpr int kMaxS = kCW * kMaxSPW;
constexpr int kMaxBL = 2;
constexpr int kXBlk = 592;  // activation block stride in shared memory (512 values + 64 B scales + pad)

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (v != v) u = 0u;  // NaN never wins (the reference's strict '>' never selects it)
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}
__device__ __forceinline__ int argmax_idx(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
}

__device__ __forceinline__ uint4 lds128(const void *p) { return *reinterpret_cast<const uint4 *>(p); }

// Build the Q8_0 activation in shared memory, block layout: block b at b*kXBlk holds its values
// (16-byte chunks in order) and then its group scales.  One thread per 32-element group.
template <int PRO>
__device__ __forceinline__ void build_activation(const GemvArgs &a, uint8_t *xsm, float *red) {
    const int tid = threadIdx.x, nthreads = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
    const int n = a.n, ng = n >> 5;
    auto put = [&](int g, const uint4 &lo, const uint4 &hi, float sc) {
        uint8_t *blk = xsm + (size_t)(g >> 4) * kXBlk;
        const int w = g & 15;
        reinterpret_cast<uint4 *>(blk + 32 * w)[0] = lo;
        reinterpret_cast<uint4 *>(blk + 32 * w)[1] = hi;
        reinterpret_cast<float *>(blk + 512)[w] = sc;
    };
    if constexpr (PRO == PRO_Q8) {
        for (int g = tid; g < ng; g += nthreads) {
            const uint4 *src = reinterpret_cast<const uint4 *>(a.xq + 32 * g);
            put(g, src[0], src[1], a.xs[g]);
        }
        return;
    } else {
        const uint8_t *erow = nullptr;
        int tok = 0;
        if constexpr (PRO == PRO_EMB_RMS) {
            tok = a.tokens[*a.pos];
            erow = a.emb + (size_t)tok * q8_row_bytes(n);
        }
        // the 32 input values of group g
        auto load_group = [&](int g, float *f) {
            if constexpr (PRO == PRO_EMB_RMS) {
                q8_packed_group(erow, n, tok, g, f);  // embedding row dequant (src/transformer.c:69)
            } else {
                const float4 *src = reinterpret_cast<const float4 *>(a.x + 32 * g);
                #pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float4 u = src[k];
                    f[4 * k] = u.x; f[4 * k + 1] = u.y; f[4 * k + 2] = u.z; f[4 * k + 3] = u.w;
                }
            }
        };
        float r = 1.0f;
        if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS) {
            float ss = 0.0f;
            for (int g = tid; g < ng; g += nthreads) {
                float f[32];
                load_group(g, f);
                if constexpr (PRO == PRO_EMB_RMS) {
                    if (blockIdx.x == 0) {  // residual stream x
                        float4 *dst = reinterpret_cast<float4 *>(const_cast<float *>(a.x) + 32 * g);
                        #pragma unroll
                        for (int k = 0; k < 8; ++k) dst[k] = make_float4(f[4 * k], f[4 * k + 1], f[4 * k + 2], f[4 * k + 3]);
                    }
                }
                #pragma unroll
                for (int k = 0; k < 32; ++k) ss = fmaf(f[k], f[k], ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float t = 0.0f;
            for (int w = 0; w < nwarps; ++w) t += red[w];
            // rmsnorm scale (src/utils.c:68-71): ss/n + 1e-5, then 1/sqrt.
            float v = __fdiv_rn(t, (float)n);
            v = __fadd_rn(v, 1e-5f);
            r = __fdiv_rn(1.0f, __fsqrt_rn(v));
        }
        for (int g = tid; g < ng; g += nthreads) {
            float f[32];
            load_group(g, f);
            if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS) {
                // o = (w*x)*scale, the reference build's evaluation order (src/utils.c:73-75)
                const float4 *wn = reinterpret_cast<const float4 *>(a.norm_w + 32 * g);
                #pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float4 u = wn[k];
                    f[4 * k] = __fmul_rn(__fmul_rn(u.x, f[4 * k]), r);
                    f[4 * k + 1] = __fmul_rn(__fmul_rn(u.y, f[4 * k + 1]), r);
                    f[4 * k + 2] = __fmul_rn(__fmul_rn(u.z, f[4 * k + 2]), r);
                    f[4 * k + 3] = __fmul_rn(__fmul_rn(u.w, f[4 * k + 3]), r);
                }
            }
            float amax = 0.0f;
            #pragma unroll
            for (int k = 0; k < 32; ++k) amax = fmaxf(amax, fabsf(f[k]));
            float sc, inv;
            q8_scale(amax, sc, inv);
            uint32_t wq[8];
            #pragma unroll
            for (int k = 0; k < 8; ++k)
                wq[k] = (uint32_t)(uint8_t)q8_round(f[4 * k], inv) |
                        ((uint32_t)(uint8_t)q8_round(f[4 * k + 1], inv) << 8) |
                        ((uint32_t)(uint8_t)q8_round(f[4 * k + 2], inv) << 16) |
                        ((uint32_t)(uint8_t)q8_round(f[4 * k + 3], inv) << 24);
            put(g, make_uint4(wq[0], wq[1], wq[2], wq[3]), make_uint4(wq[4], wq[5], wq[6], wq[7]), sc);
        }
    }
}

template <int PRO, int EPI, int BL>
__global__ void __launch_bounds__(kThreads, 2) gemv_q8_kernel(const GemvArgs a, const GemvPlan p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Q8Geom G = q8_geom(a.n);
    const int SPW = p.SPW, S = kCW * SPW;

    uint8_t *ring = smem;
    uint8_t *xsm = smem + p.xoff;
    float *red = reinterpret_cast<float *>(xsm + (size_t)G.nblk * kXBlk);
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 8);
    uint64_t *empty = full + kMaxS;
    int *flags = reinterpret_cast<int *>(empty + kMaxS);  // [0] abort [1] last CTA [2..] issued/consumed
    int *issued = flags + 2, *consumed = issued + kMaxS;
    unsigned long long *wkey = reinterpret_cast<unsigned long long *>(consumed + kMaxS);

    // rows of this CTA (for SwiGLU, whole (w1, w3) pairs)
    const int unit = (EPI == EPI_SWIGLU) ? 2 : 1;
    const int nunits = a.d / unit;
    const int r0 = (int)((long long)blockIdx.x * nunits / gridDim.x) * unit;
    const int r1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x) * unit;
    const int nst = (r1 - r0 + G.R - 1) / G.R;
    // stage k: consumer warp k % kCW, its m-th stage (m = k / kCW), slot (k % kCW)*SPW + m % SPW,
    // use number m / SPW of that slot
    auto slot_of = [&](int k) { return (k % kCW) * SPW + (k / kCW) % SPW; };
    auto use_of = [&](int k) { return (k / kCW) / SPW; };

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            issued[i] = 0;
            consumed[i] = 0;
        }
        flags[0] = 0;
        flags[1] = 0;
        mbar_fence_init();
    }
    __syncthreads();

    uint64_t policy = 0;
    auto issue = [&](int k) {  // producer lane 0 only
        const int row0 = r0 + k * G.R;
        const int rows = min(G.R, r1 - row0);
        const uint32_t bytes = (uint32_t)rows * (uint32_t)p.RS;
        const int slot = slot_of(k);
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * p.stage, a.w + (size_t)row0 * p.RS, bytes, &full[slot], policy);
        issued[slot] += 1;
    };

    if (warp == kProducer && lane == 0) {
        policy = l2_evict_first_policy();
        const int first = min(S, nst);
        for (int k = 0; k < first; ++k) issue(k);  // weights only: safe before the dependency wait
    }

    pdl_wait();
    pdl_trigger();
    build_activation<PRO>(a, xsm, red);
    __syncthreads();

    if (warp == kProducer) {
        if (lane == 0) {
            for (int k = S; k < nst; ++k) {
                const int slot = slot_of(k);
                if (*reinterpret_cast<volatile int *>(flags)) break;
                if (!mbar_wait(&empty[slot], (uint32_t)((use_of(k) - 1) & 1), a.err)) {
                    *reinterpret_cast<volatile int *>(flags) = 1;
                    break;
                }
                issue(k);
            }
        }
    } else {
        const int L = G.L;  // G.BL == BL (the launcher dispatches on it)
        const int r = lane / L, j = lane - r * L;
        const int hops = (G.nblk + BL - 1) / BL;  // segments that hold blocks
        unsigned long long best = 0ull;
        for (int k = warp; k < nst; k += kCW) {
            const int slot = slot_of(k);
            if (!mbar_wait(&full[slot], (uint32_t)(use_of(k) & 1), a.err)) {
                if (lane == 0) *reinterpret_cast<volatile int *>(flags) = 1;
                break;
            }
            if (lane == 0) consumed[slot] += 1;
            const int row0 = r0 + k * G.R;
            const int rows = min(G.R, r1 - row0);
            const int row = row0 + r;
            const bool live = r < rows;

            // ---- Phase A: products of this lane's groups, in order
            float prod[16 * BL];
            int nprod = 0;
            if (live) {
                const uint8_t *rowp = ring + (size_t)slot * p.stage + (size_t)r * p.RS;
                #pragma unroll
                for (int i = 0; i < BL; ++i) {
                    const int b = j * BL + i;
                    if (b < G.nblk) {
                        const int wb = q8_blk_width(a.n, b), ng = wb >> 5;
                        const int key = q8_swz_key(G, row, b);
                        const uint8_t *seg = rowp + q8_blk_off(b);
                        const uint8_t *xb = xsm + (size_t)b * kXBlk;
                        const float *xs = reinterpret_cast<const float *>(xb + 512);
                        #pragma unroll
                        for (int g = 0; g < 16; ++g) {
                            if (g < ng) {
                                const uint4 w0 = lds128(seg + 16 * q8_swz_q(2 * g, key, wb));
                                const uint4 w1 = lds128(seg + 16 * q8_swz_q(2 * g + 1, key, wb));
                                const uint4 x0 = lds128(xb + 32 * g), x1 = lds128(xb + 32 * g + 16);
                                const int dot = dp4a_16B(w1, x1) + dp4a_16B(w0, x0);
                                const float ws = *reinterpret_cast<const float *>(
                                    seg + wb + 16 * q8_swz_s(g >> 2, key, wb) + 4 * (g & 3));
                                prod[16 * i + g] = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, xs[g]));
                                nprod = 16 * i + g + 1;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // the stage's shared memory is free again

            // ---- Phase B: the row's ordered sum, hopping from segment j to j+1
            float carry = 0.0f;
            for (int h = 0; h < hops; ++h) {
                float s = carry;
                if (nprod == 16 * BL) {  // whole blocks: no predication in the chain
                    #pragma unroll
                    for (int q = 0; q < 16 * BL; ++q) s = __fadd_rn(s, prod[q]);
                } else {
                    #pragma unroll
                    for (int q = 0; q < 16 * BL; ++q)
                        if (q < nprod) s = __fadd_rn(s, prod[q]);
                }
                carry = __shfl_sync(FULL, s, r * L + h);
            }
            // every lane of row r now holds the row's value in `carry`
            if constexpr (EPI == EPI_SWIGLU) {
                const float h3 = __shfl_sync(FULL, carry, min(31, (r + 1) * L));
                if (live && j == 0 && !(r & 1)) {
                    // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                    float v = __fmul_rn(carry, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-carry))));
                    v = __fmul_rn(v, h3);
                    a.out[row >> 1] = v;
                }
            } else if (live && j == 0) {
                if constexpr (EPI == EPI_ADD) a.out[row] = __fadd_rn(a.out[row], carry);
                else a.out[row] = carry;
                if constexpr (EPI == EPI_ARGMAX) {
                    const unsigned long long key = argmax_key(carry, row);
                    best = key > best ? key : best;
                }
            }
        }
        if constexpr (EPI == EPI_ARGMAX) {
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(FULL, best, o);
                best = other > best ? other : best;
            }
            if (lane == 0) wkey[warp] = best;
        }
    }
    __syncthreads();

    // Error path only: never leave a bulk copy in flight into shared memory of an exiting CTA.
    if (tid == 0 && *reinterpret_cast<volatile int *>(flags)) {
        for (int i = 0; i < S; ++i) {
            while (consumed[i] < issued[i]) {
                if (!mbar_wait(&full[i], (uint32_t)(consumed[i] & 1), a.err)) break;
                consumed[i] += 1;
            }
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kCW; ++w) b = wkey[w] > b ? wkey[w] : b;
            a.amax_part[blockIdx.x] = b;
            __threadfence();
            const unsigned ticket = atomicAdd(a.amax_count, 1u);
            flags[1] = (ticket == gridDim.x - 1);
        }
        __syncthreads();
        if (flags[1] && tid == 0) {
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

template <int PRO, int EPI, int BL>
cudaError_t launch_bl(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    auto kern = gemv_q8_kernel<PRO, EPI, BL>;
    // Opt in to the dynamic shared memory this launch needs (raised monotonically, per device).
    static int attr_bytes[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (attr_bytes[dev] < (int)p.smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
        if (e != cudaSuccess) return e;
        attr_bytes[dev] = (int)p.smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, p);
}

template <int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    return q8_geom(a.n).BL == 1 ? launch_bl<PRO, EPI, 1>(a, p, st, pdl) : launch_bl<PRO, EPI, 2>(a, p, st, pdl);
}

}  // namespace

size_t gemv_x_bytes(int n) { return (size_t)q8_geom(n).nblk * kXBlk; }

bool gemv_supported(int n, int d, int epi) {
    if (n <= 0 || d <= 0 || n % 32) return false;
    const Q8Geom g = q8_geom(n);
    if (g.BL > kMaxBL) return false;  // n > 32768
    if (epi == EPI_SWIGLU && ((g.R & 1) || (d & 1))) return false;
    return true;
}

GemvPlan plan_gemv(int n, int d, int epi, int num_sms, int ctas_per_sm, size_t smem_budget) {
    GemvPlan p;
    const Q8Geom g = q8_geom(n);
    p.RS = (int)q8_row_bytes(n);
    const int unit = epi == EPI_SWIGLU ? 2 : 1;
    const size_t tail = gemv_x_bytes(n) + 32 + kMaxS * 16 + 8 + kMaxS * 8 + kCW * 8 + 64;
    const int cps = ctas_per_sm == 2 ? 2 : 1;
    const size_t per_sm = smem_budget ? smem_budget : 220 * 1024;
    const size_t per_cta = std::min((size_t)227 * 1024, per_sm / cps - 1024);
    p.grid = std::max(1, std::min(cps * num_sms, d / unit));
    const int rows_per_cta = (d / unit + p.grid - 1) / p.grid * unit;
    p.stage = ((size_t)std::min(g.R, rows_per_cta) * p.RS + 127) & ~(size_t)127;
    p.CW = kCW;
    const int nst = (rows_per_cta + g.R - 1) / g.R;
    int spw = kMaxSPW;
    while (spw > 1 && ((size_t)kCW * spw * p.stage + tail > per_cta || kCW * (spw - 1) >= nst)) --spw;
    p.SPW = spw;
    p.ring = (size_t)kCW * spw * p.stage;
    p.xoff = p.ring;
    p.smem = p.ring + tail;
    return p;
}

cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    if (!gemv_supported(a.n, a.d, a.epi) || p.smem > 227 * 1024 || p.CW != kCW || p.SPW < 1 || p.SPW > kMaxSPW)
        return cudaErrorInvalidValue;
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
