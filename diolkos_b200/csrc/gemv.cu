// gemv.cu -- the batch-1 Q8_0 GEMV (reference matmul_Q8_0, src/utils.c:106-138) for sm_100a.
//
// Weights are in the packed tile layout (dk_kernels.h): tiles of T rows (T chosen so that every SM
// owns the same number of rows), each tile stored block by block, so that one STAGE -- the 512-column
// block b of the T rows of one tile -- is one contiguous range of T row segments (about 16-18 KB for
// the LLaMA shapes).
//
// Persistent kernel, one CTA per SM; CTA c owns a contiguous range of tiles.  Warp 4 is the
// producer: it streams stages with the bulk-copy engine (cp.async.bulk, one copy per stage,
// completion counted on an mbarrier, L2 evict-first) into per-consumer rings in shared memory and
// keeps PF further stages prefetched into L2 (cp.async.bulk.prefetch.L2).  The shared-memory
// footprint stays near 100 KB so that the next kernel's CTA fits beside this one.  The first stages
// and prefetches are issued BEFORE griddepcontrol.wait, i.e. while the previous kernel in the stream
// is still running: weights never depend on it.
//
// Consumers: warp w takes the CTA's tiles w, w+CW, ...; LANE r OF THE WARP IS ROW r OF THE TILE.
// For each stage the lane walks its row's 16 groups in order: exact int32 dot (dp4a against the
// broadcast activation), then sum = sum + (float)dot * (w_scale * x_scale) with no FMA -- the
// order and rounding of the reference's compiled loop, so the output is bit-identical to the
// reference build.  The sum is carried in a register from block to block.  Only the warp that owns
// a ring slot ever waits on it, so the mbarrier phases of a slot are always waited in order.  All
// hot-loop loads are explicit ld.shared on 32-bit shared addresses.
#include "dk_common.cuh"
#include "dk_kernels.h"

#include <algorithm>
#include <cmath>

namespace dk {
namespace {

constexpr int kThreads = 160;  // warps 0..3 consume, warp 4 produces; all build the activation
constexpr int kProducer = 4;
constexpr int kMaxCW = 4;
constexpr int kMaxSPW = 4;
constexpr int kMaxSlots = kMaxCW * kMaxSPW;
constexpr size_t kSmemBudget = 104 * 1024;    // two of these fit on an SM (this kernel + the next)
constexpr size_t kPrefetchBytes = 40 * 1024;  // L2 prefetch distance ahead of the rings, per CTA

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (v != v) u = 0u;  // NaN never wins (the reference's strict '>' never selects it)
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}
__device__ __forceinline__ int argmax_idx(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
}

// Build the Q8_0 activation in shared memory: xq int8[n] then xs fp32[n/32].  One thread per
// 32-element group.
template <int PRO>
__device__ __forceinline__ void build_activation(const GemvArgs &a, int8_t *xq, float *xs, float *red) {
    const int tid = threadIdx.x, nthreads = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
    const int n = a.n, ng = n >> 5;
    if constexpr (PRO == PRO_Q8) {
        for (int i = tid; i < n / 16; i += nthreads)
            reinterpret_cast<uint4 *>(xq)[i] = reinterpret_cast<const uint4 *>(a.xq)[i];
        for (int g = tid; g < ng; g += nthreads) xs[g] = a.xs[g];
        return;
    } else {
        int tok = 0;
        if constexpr (PRO == PRO_EMB_RMS) tok = a.tokens[*a.pos];
        auto load_group = [&](int g, float *f) {
            if constexpr (PRO == PRO_EMB_RMS) {
                q8_packed_group(a.emb, n, a.emb_T, tok, g, f);  // embedding row dequant (src/transformer.c:69)
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
            reinterpret_cast<uint4 *>(xq + 32 * g)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
            reinterpret_cast<uint4 *>(xq + 32 * g)[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
            xs[g] = sc;
        }
    }
}

// One lane's reference-order sum over one block of its row (FULL: 512 columns).  seg, xq, xs are
// 32-bit shared-memory addresses of the row's segment and of this block's activation values/scales.
template <bool FULL>
__device__ __forceinline__ float block_chain(float sum, uint32_t seg, uint32_t xq, uint32_t xs, int wb, int r) {
    const int ng = FULL ? 16 : (wb >> 5);
    const int cw = FULL ? 512 : wb;
    const uint32_t scp = seg + cw;
    #pragma unroll 4
    for (int g4 = 0; g4 < ng; g4 += 4) {
        const uint4 s4 = lds128(scp + 16 * q8_swz_s(g4 >> 2, r, cw));
        const float wsc[4] = {__uint_as_float(s4.x), __uint_as_float(s4.y), __uint_as_float(s4.z),
                              __uint_as_float(s4.w)};
        const float4 x4 = lds_f4(xs + 4 * g4);
        const float xsc[4] = {x4.x, x4.y, x4.z, x4.w};
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int g = g4 + j;
            if (!FULL && g >= ng) break;
            const uint4 w0 = lds128(seg + 16 * q8_swz_q(2 * g, r, cw));
            const uint4 w1 = lds128(seg + 16 * q8_swz_q(2 * g + 1, r, cw));
            const uint4 x0 = lds128(xq + 32 * g), x1 = lds128(xq + 32 * g + 16);
            const int dot = dp4a_16B(w1, x1) + dp4a_16B(w0, x0);
            sum = __fadd_rn(sum, __fmul_rn(__int2float_rn(dot), __fmul_rn(wsc[j], xsc[j])));
        }
    }
    return sum;
}

struct Sched {  // which stages exist, and where they come from
    int t0, nt, CW, nblk, T, n;
    size_t tile_bytes;
    __device__ int nstages(int w) const { return nt > w ? ((nt - w + CW - 1) / CW) * nblk : 0; }
    __device__ int tile_of(int w, int k) const { return t0 + w + CW * (k / nblk); }
    __device__ const uint8_t *src(const uint8_t *base, int w, int k) const {
        return base + (size_t)tile_of(w, k) * tile_bytes + (size_t)T * 576 * (k % nblk);
    }
    __device__ uint32_t bytes(int k) const { return (uint32_t)((size_t)T * q8_blk_bytes(q8_blk_width(n, k % nblk))); }
};

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_q8_kernel(const GemvArgs a, const GemvPlan p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = a.n;

    uint8_t *ring = smem;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + p.xoff);
    float *xs = reinterpret_cast<float *>(smem + p.xoff + ((n + 15) & ~15));
    float *red = xs + ((n / 32 + 3) & ~3);
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 8);
    uint64_t *empty = full + kMaxSlots;
    int *flags = reinterpret_cast<int *>(empty + kMaxSlots);  // [0] abort, [1] last CTA
    int *issued = flags + 2, *consumed = issued + kMaxSlots;
    unsigned long long *wkey = reinterpret_cast<unsigned long long *>(consumed + kMaxSlots);
    const uint32_t ring_s = smem_u32(ring), xq_s = smem_u32(xq), xs_s = smem_u32(xs);

    Sched sc;
    sc.t0 = (int)((long long)blockIdx.x * p.ntiles / gridDim.x);
    sc.nt = (int)((long long)(blockIdx.x + 1) * p.ntiles / gridDim.x) - sc.t0;
    sc.CW = p.CW;
    sc.nblk = (n + 511) >> 9;
    sc.T = p.T;
    sc.n = n;
    sc.tile_bytes = (size_t)p.T * q8_row_bytes(n);
    const int SPW = p.SPW, CW = p.CW;
    // Stage k of consumer warp w: its tile w + CW*(k / nblk), block k % nblk; slot w*SPW + k % SPW,
    // use k / SPW of that slot.  The producer walks the stages round-robin over the warps.
    const int kmax = sc.nstages(0);  // warp 0 has the most stages

    if (tid == 0) {
        for (int i = 0; i < CW * SPW; ++i) {
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
    if (warp == kProducer && lane == 0) {
        // Weights only, so safe before the dependency wait: fill every ring slot, then prefetch the
        // next PF stages of each warp into L2.
        policy = l2_evict_first_policy();
        for (int k = 0; k < min(SPW, kmax); ++k)
            for (int w = 0; w < CW; ++w) {
                if (k >= sc.nstages(w)) continue;
                const int slot = w * SPW + k;
                mbar_arrive_expect_tx(&full[slot], sc.bytes(k));
                bulk_g2s(ring + (size_t)slot * p.slot, sc.src(a.w, w, k), sc.bytes(k), &full[slot], policy);
                issued[slot] += 1;
            }
        for (int k = SPW; k < min(SPW + p.PF, kmax); ++k)
            for (int w = 0; w < CW; ++w)
                if (k < sc.nstages(w)) bulk_prefetch_l2(sc.src(a.w, w, k), sc.bytes(k));
    }

    pdl_wait();
    pdl_trigger();
    build_activation<PRO>(a, xq, xs, red);
    __syncthreads();

    if (warp == kProducer) {
        if (lane == 0) {
            bool stop = false;
            for (int k = SPW; k < kmax && !stop; ++k) {
                for (int w = 0; w < CW; ++w) {
                    if (k >= sc.nstages(w)) continue;
                    const int slot = w * SPW + (k % SPW);
                    if (*reinterpret_cast<volatile int *>(flags) ||
                        !mbar_wait(&empty[slot], (uint32_t)(((k / SPW) - 1) & 1), a.err)) {
                        *reinterpret_cast<volatile int *>(flags) = 1;
                        stop = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[slot], sc.bytes(k));
                    bulk_g2s(ring + (size_t)slot * p.slot, sc.src(a.w, w, k), sc.bytes(k), &full[slot], policy);
                    issued[slot] += 1;
                    const int kp = k + p.PF;  // keep the L2 prefetch PF stages ahead
                    if (kp < sc.nstages(w)) bulk_prefetch_l2(sc.src(a.w, w, kp), sc.bytes(kp));
                }
            }
        }
    } else if (warp < CW) {
        const int w = warp, ns = sc.nstages(w);
        unsigned long long best = 0ull;
        float sum = 0.0f;
        for (int k = 0; k < ns; ++k) {
            const int slot = w * SPW + (k % SPW);
            if (!mbar_wait(&full[slot], (uint32_t)((k / SPW) & 1), a.err)) {
                if (lane == 0) *reinterpret_cast<volatile int *>(flags) = 1;
                break;
            }
            if (lane == 0) consumed[slot] += 1;
            const int b = k % sc.nblk;
            const int row = sc.tile_of(w, k) * p.T + lane;
            const bool live = lane < p.T && row < a.d;
            if (b == 0) sum = 0.0f;
            const int wb = q8_blk_width(n, b);
            if (live) {
                const uint32_t seg = ring_s + (uint32_t)(slot * p.slot + lane * q8_blk_bytes(wb));
                const uint32_t xqb = xq_s + 512u * b, xsb = xs_s + 64u * b;
                if (wb == 512) sum = block_chain<true>(sum, seg, xqb, xsb, 512, lane);
                else sum = block_chain<false>(sum, seg, xqb, xsb, wb, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (b == sc.nblk - 1) {  // the tile's rows are finished
                if constexpr (EPI == EPI_SWIGLU) {
                    const float h3 = __shfl_down_sync(FULL, sum, 1);
                    if (live && !(lane & 1)) {
                        // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                        float v = __fmul_rn(sum, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-sum))));
                        v = __fmul_rn(v, h3);
                        a.out[row >> 1] = v;
                    }
                } else if (live) {
                    if constexpr (EPI == EPI_ADD) a.out[row] = __fadd_rn(a.out[row], sum);
                    else a.out[row] = sum;
                    if constexpr (EPI == EPI_ARGMAX) {
                        const unsigned long long key = argmax_key(sum, row);
                        best = key > best ? key : best;
                    }
                }
            }
        }
        if constexpr (EPI == EPI_ARGMAX) {
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(FULL, best, o);
                best = other > best ? other : best;
            }
            if (lane == 0) wkey[w] = best;
        }
    }
    __syncthreads();

    // Error path only: never leave a bulk copy in flight into shared memory of an exiting CTA.
    if (tid == 0 && *reinterpret_cast<volatile int *>(flags)) {
        for (int i = 0; i < CW * SPW; ++i) {
            while (consumed[i] < issued[i]) {
                if (!mbar_wait(&full[i], (uint32_t)(consumed[i] & 1), a.err)) break;
                consumed[i] += 1;
            }
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < CW; ++w) b = wkey[w] > b ? wkey[w] : b;
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

template <int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    auto kern = gemv_q8_kernel<PRO, EPI>;
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

}  // namespace

size_t gemv_x_bytes(int n) { return (((size_t)n + 15) & ~(size_t)15) + (size_t)((n / 32 + 3) & ~3) * 4; }

int gemv_tile_rows(int d, int epi, int num_sms) { return q8_tile_rows(d, num_sms, epi == EPI_SWIGLU ? 2 : 1); }

bool gemv_supported(int n, int d, int epi) {
    if (n <= 0 || d <= 0 || n % 32) return false;
    if (epi == EPI_SWIGLU && (d & 1)) return false;
    return gemv_x_bytes(n) + 36 * 1024 < kSmemBudget;  // the activation must fit beside one ring slot
}

GemvPlan plan_gemv(int n, int d, int epi, int num_sms) {
    GemvPlan p;
    p.T = gemv_tile_rows(d, epi, num_sms);
    p.ntiles = (d + p.T - 1) / p.T;
    p.grid = std::max(1, std::min(num_sms, p.ntiles));
    const int tiles_per_cta = (p.ntiles + p.grid - 1) / p.grid;
    const int nblk = (n + 511) / 512;
    p.CW = std::max(1, std::min(kMaxCW, tiles_per_cta));
    p.slot = (size_t)p.T * q8_blk_bytes(std::min(n, 512));
    const size_t tail = gemv_x_bytes(n) + 32 + kMaxSlots * 16 + 8 + kMaxSlots * 8 + kMaxCW * 8 + 64;
    const int stages_per_warp = ((tiles_per_cta + p.CW - 1) / p.CW) * nblk;
    int spw = kMaxSPW;
    while (spw > 1 && ((size_t)p.CW * spw * p.slot + tail > kSmemBudget || spw > stages_per_warp)) --spw;
    p.SPW = spw;
    p.PF = (int)(kPrefetchBytes / ((size_t)p.CW * p.slot));
    p.xoff = (size_t)p.CW * spw * p.slot;
    p.smem = p.xoff + tail;
    return p;
}

cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    if (!gemv_supported(a.n, a.d, a.epi) || p.smem > 227 * 1024 || p.CW < 1 || p.CW > kMaxCW || p.SPW < 1 ||
        p.SPW > kMaxSPW || p.T < 1 || p.T > 32)
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
