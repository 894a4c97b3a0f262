// gemv.cu -- the batch-1 Q8_0 GEMV (reference matmul_Q8_0, src/utils.c:106-138) for sm_100a.
//
// Weights are in the packed tile layout (dk_kernels.h): tiles of T rows (T chosen so that every SM
// owns the same number of rows), each tile stored block by block, so that one STAGE -- the 512-column
// block b of the T rows of one tile -- is one contiguous range of T row segments (about 16-18 KB for
// the LLaMA shapes).
//
// Persistent kernel, one CTA per SM; CTA c owns a contiguous range of tiles, i.e. a sequence of
// stages (its tiles in order, each tile's blocks in order).  NP producer threads (in separate warps:
// under load the copy engine completes only a few copies per microsecond for each issuing thread)
// stream the stages with the bulk-copy engine (cp.async.bulk, one copy per stage, completion counted on the slot's
// mbarrier, L2 evict-first) through a ring of S shared-memory slots; the first S copies are issued
// BEFORE griddepcontrol.wait, i.e. while the previous kernel in the stream is still running (weights
// never depend on it).  Shared memory stays near 100 KB and registers at 128 per thread, so the next
// kernel's CTA fits beside this one.
//
// NC consumer warps take the stages round-robin; LANE r OF A WARP IS ROW r OF THE TILE.  For its
// stage a lane computes the row's 16 group terms (float)dot * (w_scale * x_scale) -- the exact int32
// dot with dp4a against the broadcast activation, the products rounded as in the reference -- then
// adds them to the row's running sum in group order, sum = sum + term with no FMA.  The running sums
// travel from the warp of stage s to the warp of stage s+1 through shared memory, so the additions
// of every row happen in the reference's order while the dot products of NC stages proceed in
// parallel: the output is bit-identical to the reference build.  All hot-loop loads are explicit
// ld.shared on 32-bit shared addresses.
#include "dk_common.cuh"
#include "dk_kernels.h"
#include "gemv_core.cuh"

#include <algorithm>
#include <cstdlib>
#include <cmath>

namespace dk {
namespace {

constexpr int kMaxConsumers = 6;
constexpr int kMinWarps = 8;   // warps launched per CTA (consumers + producer + helpers for the activation)
constexpr int kMaxSlots = 16;
constexpr size_t kSmemBudget = 112 * 1024;    // two of these fit on an SM (228 KB: this kernel + the next, or a batch's two CTA groups)
constexpr int kPrefetchStages = 3;           // L2 prefetch distance beyond the ring, in stages

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
        if constexpr (PRO == PRO_RMS_REDUCE) {
            // Every rank's partial rows for this exchange point have landed in this rank's receive
            // area once its counter reaches the target; then every thread reads them from L2.
            if (tid == 0) {
                const unsigned long long target =
                    (*a.epoch * (unsigned long long)a.red_period + (unsigned long long)a.red_index + 1ull) *
                    (unsigned long long)a.tp_world * (unsigned long long)n;
                wait_counter(a.cnt, target, a.err);
            }
            __syncthreads();
            __threadfence();
        }
        auto load_group = [&](int g, float *f) {
            if constexpr (PRO == PRO_EMB_RMS) {
                q8_packed_group(a.emb, n, a.emb_T, tok, g, f);  // embedding row dequant (src/transformer.c:69)
            } else if constexpr (PRO == PRO_RMS_REDUCE) {
                // x + (partial_0 + partial_1 + ...), ranks in order: the same bits on every rank.
                // (L2 loads: this kernel skips the dependency wait.)
                const float4 *src = reinterpret_cast<const float4 *>(a.x + 32 * g);
                #pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float4 t = __ldcg(reinterpret_cast<const float4 *>(a.recv + 32 * g) + k);
                    for (int q = 1; q < a.tp_world; ++q) {
                        const float4 u = __ldcg(reinterpret_cast<const float4 *>(a.recv + (size_t)q * n + 32 * g) + k);
                        t = make_float4(__fadd_rn(t.x, u.x), __fadd_rn(t.y, u.y), __fadd_rn(t.z, u.z), __fadd_rn(t.w, u.w));
                    }
                    const float4 x = __ldcg(src + k);
                    f[4 * k] = __fadd_rn(x.x, t.x); f[4 * k + 1] = __fadd_rn(x.y, t.y);
                    f[4 * k + 2] = __fadd_rn(x.z, t.z); f[4 * k + 3] = __fadd_rn(x.w, t.w);
                }
            } else {
                const float4 *src = reinterpret_cast<const float4 *>(a.x + 32 * g);
                #pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float4 u = src[k];
                    f[4 * k] = u.x; f[4 * k + 1] = u.y; f[4 * k + 2] = u.z; f[4 * k + 3] = u.w;
                }
            }
        };
        // The first group of each thread stays in registers between the two passes (with n <= 32 *
        // threads that is every group, so x is read once).
        float f0[32];
        if (tid < ng) load_group(tid, f0);
        float r = 1.0f;
        if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS || PRO == PRO_RMS_REDUCE) {
            float ss = 0.0f;
            for (int g = tid; g < ng; g += nthreads) {
                float f[32];
                if (g == tid) {
                    #pragma unroll
                    for (int k = 0; k < 32; ++k) f[k] = f0[k];
                } else {
                    load_group(g, f);
                }
                if constexpr (PRO == PRO_EMB_RMS || PRO == PRO_RMS_REDUCE) {
                    if (blockIdx.x == 0) {  // residual stream x (the reduce writes a second buffer)
                        float4 *dst = reinterpret_cast<float4 *>((PRO == PRO_RMS_REDUCE ? a.x_out : const_cast<float *>(a.x)) + 32 * g);
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
            if (g == tid) {
                #pragma unroll
                for (int k = 0; k < 32; ++k) f[k] = f0[k];
            } else {
                load_group(g, f);
            }
            if constexpr (PRO == PRO_RMS || PRO == PRO_EMB_RMS || PRO == PRO_RMS_REDUCE) {
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

// Fast prologue for the rmsnorm family when n == 16 * threads (e.g. dim 4096 on 256 threads): thread t
// owns the 16 values [16t, 16t+16), half of group t/2, so every thread loads at once and one memory
// round trip brings the whole activation in.  nw = this thread's 16 norm weights, loaded before the
// dependency wait (weights are constant).  PRO_RMS_REDUCE adds the ranks' partials (rank order) and
// CTA 0 stores the new residual; then rmsnorm, and the two threads of a group agree on its Q8_0 scale.
template <int PRO>
__device__ __forceinline__ void build_activation_half(const GemvArgs &a, int8_t *xq, float *xs, float *red,
                                                      const float4 (&nw)[4]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    const int n = a.n, e0 = 16 * tid;
    float4 v[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = __ldcg(reinterpret_cast<const float4 *>(a.x + e0) + k);
    if constexpr (PRO == PRO_RMS_REDUCE) {
        // Every rank's partial rows for this exchange point are in this rank's receive area once its
        // counter reaches the target.
        if (tid == 0) {
            const unsigned long long target =
                (*a.epoch * (unsigned long long)a.red_period + (unsigned long long)a.red_index + 1ull) *
                (unsigned long long)a.tp_world * (unsigned long long)n;
            wait_counter(a.cnt, target, a.err);
        }
        __syncthreads();
        __threadfence();
        // x + (partial_0 + partial_1 + ...), ranks in order: the same bits on every rank.  Two ranks'
        // loads are in flight at a time.
        float4 t[4];
        #pragma unroll
        for (int k = 0; k < 4; ++k) t[k] = __ldcg(reinterpret_cast<const float4 *>(a.recv + e0) + k);
        for (int q = 1; q < a.tp_world; q += 2) {
            float4 u[4], w[4];
            const bool two = q + 1 < a.tp_world;
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                u[k] = __ldcg(reinterpret_cast<const float4 *>(a.recv + (size_t)q * n + e0) + k);
                w[k] = two ? __ldcg(reinterpret_cast<const float4 *>(a.recv + (size_t)(q + 1) * n + e0) + k)
                           : make_float4(0, 0, 0, 0);
            }
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                t[k] = make_float4(__fadd_rn(t[k].x, u[k].x), __fadd_rn(t[k].y, u[k].y), __fadd_rn(t[k].z, u[k].z),
                                   __fadd_rn(t[k].w, u[k].w));
                if (two)
                    t[k] = make_float4(__fadd_rn(t[k].x, w[k].x), __fadd_rn(t[k].y, w[k].y),
                                       __fadd_rn(t[k].z, w[k].z), __fadd_rn(t[k].w, w[k].w));
            }
        }
        #pragma unroll
        for (int k = 0; k < 4; ++k)
            v[k] = make_float4(__fadd_rn(v[k].x, t[k].x), __fadd_rn(v[k].y, t[k].y), __fadd_rn(v[k].z, t[k].z),
                               __fadd_rn(v[k].w, t[k].w));
        if (blockIdx.x == 0) {
            #pragma unroll
            for (int k = 0; k < 4; ++k) reinterpret_cast<float4 *>(a.x_out + e0)[k] = v[k];
        }
    }
    float f[16];
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
        f[4 * k] = v[k].x; f[4 * k + 1] = v[k].y; f[4 * k + 2] = v[k].z; f[4 * k + 3] = v[k].w;
    }
    float ss = 0.0f;
    #pragma unroll
    for (int k = 0; k < 16; ++k) ss = fmaf(f[k], f[k], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < nwarps; ++w) tot += red[w];
    // rmsnorm scale (src/utils.c:68-71): ss/n + 1e-5, then 1/sqrt; o = (w*x)*scale (:73-75)
    float r = __fdiv_rn(tot, (float)n);
    r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(r, 1e-5f)));
    float amax = 0.0f;
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
        f[4 * k] = __fmul_rn(__fmul_rn(nw[k].x, f[4 * k]), r);
        f[4 * k + 1] = __fmul_rn(__fmul_rn(nw[k].y, f[4 * k + 1]), r);
        f[4 * k + 2] = __fmul_rn(__fmul_rn(nw[k].z, f[4 * k + 2]), r);
        f[4 * k + 3] = __fmul_rn(__fmul_rn(nw[k].w, f[4 * k + 3]), r);
    }
    #pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(f[k]));
    amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 1));  // the group's other half
    float sc, inv;
    q8_scale(amax, sc, inv);
    uint32_t wq[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k)
        wq[k] = (uint32_t)(uint8_t)q8_round(f[4 * k], inv) | ((uint32_t)(uint8_t)q8_round(f[4 * k + 1], inv) << 8) |
                ((uint32_t)(uint8_t)q8_round(f[4 * k + 2], inv) << 16) |
                ((uint32_t)(uint8_t)q8_round(f[4 * k + 3], inv) << 24);
    reinterpret_cast<uint4 *>(xq + e0)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
    if (!(tid & 1)) xs[tid >> 1] = sc;
}

// Block layout (warps): 0 .. NC-1 consume, NC .. NC+NP-1 produce (one thread each), the rest (up to
// kMinWarps) only help build the activation.  Stage s of the CTA sits in ring slot s % S and is consumed by warp s % NC.  A
// consumer computes its stage's per-group terms as soon as the data is in, frees the slot, then
// waits for the running row sums of stage s-1 (the TOKEN, passed warp to warp through shared
// memory), folds its 16 terms into them in group order and passes them on to the warp of stage s+1.
// So the fp32 additions of every row happen in exactly the reference's order, while the dot
// products of consecutive stages run on different warps at the same time.  The token travels along
// ALL stages of the CTA (across tile boundaries too, where the sums restart at 0), so a warp is never
// handed a second token before it has taken the first.
template <int PRO, int EPI>
__global__ void __launch_bounds__(32 * kMinWarps, 2) gemv_q8_kernel(const GemvArgs a, const GemvPlan p,
                                                                     const GemvBatch bt) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = a.n, NC = p.NW, S = p.S;

    uint8_t *ring = smem;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + p.xoff);
    float *xs = reinterpret_cast<float *>(smem + p.xoff + ((n + 15) & ~15));
    float *red = xs + ((n / 32 + 3) & ~3);                           // [kMinWarps]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + kMinWarps);  // [kMaxSlots]
    uint64_t *empty = full + kMaxSlots;                              // [kMaxSlots]
    // running row sums handed to each consumer warp: per lane one word = (stage index << 32) | sum bits
    unsigned long long *tok = reinterpret_cast<unsigned long long *>(empty + kMaxSlots);  // [kMaxConsumers][32]
    unsigned long long *wkey = tok + kMaxConsumers * 32;
    int *flags = reinterpret_cast<int *>(wkey + kMaxConsumers);      // [0] abort, [1] last CTA
    const uint32_t ring_s = smem_u32(ring), xq_s = smem_u32(xq), xs_s = smem_u32(xs);

    // A batch's CTA groups cover the same tiles: CTA index within the group, and the group
    const int cgrid = bt.count > 0 ? p.grid : (int)gridDim.x;
    const int cidx = (int)blockIdx.x % cgrid, grp = (int)blockIdx.x / cgrid;
    Sched sc;
    sc.t0 = (int)((long long)cidx * p.ntiles / cgrid);
    sc.nt = (int)((long long)(cidx + 1) * p.ntiles / cgrid) - sc.t0;
    sc.nblk = (n + 511) >> 9;
    sc.T = p.T;
    sc.n = n;
    sc.nst = sc.nt * sc.nblk;
    sc.tile_bytes = (size_t)p.T * q8_row_bytes(n);
    // A batch (bt.count matrices of the same shape): this CTA's stages of its group's matrices -- k-th
    // matrix grp + k * groups -- one after another in one sequence, so the ring streams from one matrix
    // into the next.
    const int G = bt.count > 0 ? bt.groups : 1;
    const int nmat = bt.count > 0 ? (bt.count - grp + G - 1) / G : 1;
    const int total = nmat * sc.nst;
    auto wsrc = [&](int s) -> const uint8_t * {
        if (bt.count == 0) return sc.src(a.w, s);
        const int k = s / sc.nst;
        return sc.src(bt.w[grp + k * G], s - k * sc.nst);
    };

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < NC * 32; ++i) tok[i] = 0xFFFFFFFF00000000ull;  // tag -1
        flags[0] = 0;
        flags[1] = 0;
        mbar_fence_init();
    }
    __syncthreads();

    // Producer warps NC .. NC+NP-1: producer q issues the stages s = q (mod NP), into the slots
    // s % S (S is a multiple of NP, so each slot has one producer).  Weights only, so the ring is filled
    // (and PF more stages are prefetched into L2) before the dependency wait.
    const int NP = p.NP, q = warp - NC;
    const bool producer = q >= 0 && q < NP && lane == 0;
    uint64_t policy = 0;
    int next = q;  // this producer's next stage to issue
    if (producer) {
        policy = l2_evict_first_policy();
        for (; next < min(S, total); next += NP) {
            mbar_arrive_expect_tx(&full[next], sc.bytes(next));
            bulk_g2s(ring + (size_t)next * p.slot, wsrc(next), sc.bytes(next), &full[next], policy);
        }
        for (int s = S + q; s < min(S + p.PF, total); s += NP) bulk_prefetch_l2(wsrc(s), sc.bytes(s));
    }

    // The rmsnorm family on n == 16 * threads takes the one-round-trip prologue; its norm weights are
    // constant, so they are loaded before the dependency wait.
    constexpr bool kRmsFamily = PRO == PRO_RMS || PRO == PRO_RMS_REDUCE;
    const bool half = kRmsFamily && n == 16 * (int)blockDim.x;
    float4 nw[4];
    if (half) {
        #pragma unroll
        for (int k = 0; k < 4; ++k) nw[k] = __ldg(reinterpret_cast<const float4 *>(a.norm_w + 16 * tid) + k);
    }
    // A tensor-parallel reduce GEMV does not wait for the previous kernel: its new input (the ranks'
    // partial rows) is announced by the exchange counter, and everything else it reads or overwrites
    // was last written or read by kernels that an earlier kernel of the step already waited for.  So
    // it starts on the partials as soon as the last rank's rows land, not when the producing kernel's
    // last CTA has drained its fence and exited.
    // A batch's later GEMV (early_input) reads only weights and an input that was complete before the
    // previous kernel started: it waits for that kernel only before its first output store (below).
    const bool early = PRO == PRO_F32 && EPI == EPI_STORE && a.early_input;
    if constexpr (PRO != PRO_RMS_REDUCE) {
        if (!early) pdl_wait();
    }
    pdl_trigger();
    if (half) {
        if constexpr (kRmsFamily) build_activation_half<PRO>(a, xq, xs, red, nw);
    } else {
        build_activation<PRO>(a, xq, xs, red);
    }
    __syncthreads();

    if (q >= 0 && q < NP) {
        if (lane == 0) {
            for (; next < total; next += NP) {
                const int slot = next % S;
                if (!mbar_wait_abortable(&empty[slot], (uint32_t)(((next / S) - 1) & 1), a.err, flags, false)) {
                    flags[0] = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], sc.bytes(next));
                bulk_g2s(ring + (size_t)slot * p.slot, wsrc(next), sc.bytes(next), &full[slot], policy);
                if (next + p.PF < total) bulk_prefetch_l2(wsrc(next + p.PF), sc.bytes(next + p.PF));
            }
            // Never leave a copy in flight into the shared memory of an exiting CTA: each of this
            // producer's slots has at most one outstanding copy, the last one issued into it.
            for (int last = next - NP; last >= q && last >= next - S; last -= NP)
                mbar_wait(&full[last % S], (uint32_t)((last / S) & 1), a.err);
        }
    } else if (warp < NC) {
        const int c = warp;
        unsigned long long best = 0ull;
        bool waited = !early;  // the dependency wait before this thread's first output store
        for (int s = c; s < total; s += NC) {
            const int slot = s % S;
            const int k = s / sc.nst;                   // this CTA's k-th matrix of the batch
            const int m = bt.count > 0 ? grp + k * G : 0;  // its index in the batch (0 without a batch)
            if (!__all_sync(FULL, mbar_wait_abortable(&full[slot], (uint32_t)((s / S) & 1), a.err, flags, false))) {
                if (lane == 0) flags[0] = 1;
                break;
            }
            const int b = s % sc.nblk;
            const int row = (sc.t0 + (s - k * sc.nst) / sc.nblk) * p.T + lane;
            const bool live = lane < p.T && row < a.d;
            const int wb = q8_blk_width(n, b);
            float t[16] = {};
            if (live) {
                const uint32_t seg = ring_s + (uint32_t)(slot * p.slot + lane * q8_blk_bytes(wb));
                const uint32_t xqb = xq_s + 512u * b, xsb = xs_s + 64u * b;
                if (wb == 512) block_terms_full(t, seg, xqb, xsb, lane);
                else block_terms_part(t, seg, xqb, xsb, wb, lane);
                // Pin the terms here: without this the compiler may sink their arithmetic past the
                // token wait below, onto the serial path that the hand-off is meant to keep short.
                #pragma unroll
                for (int g = 0; g < 16; ++g) asm volatile("" : "+f"(t[g]));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            float sum = 0.0f;
            if (s > 0) {  // the running sum of this lane's row after stage s-1
                float prev = 0.0f;
                if (!__all_sync(FULL, lane_token_wait(&tok[c * 32], lane, s, prev, a.err, flags))) {
                    if (lane == 0) flags[0] = 1;
                    break;
                }
                if (b > 0) sum = prev;
            }
            if (live) {
                if (wb == 512) {
                    #pragma unroll
                    for (int g = 0; g < 16; ++g) sum = __fadd_rn(sum, t[g]);
                } else {
                    #pragma unroll
                    for (int g = 0; g < 16; ++g)
                        if (g < (wb >> 5)) sum = __fadd_rn(sum, t[g]);
                }
            }
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
                    if constexpr (EPI == EPI_ADD) {
                        a.out[row] = __fadd_rn(a.out[row], sum);
                    } else if constexpr (EPI == EPI_PEER) {
                        // This rank's partial of row `row`, into every rank's receive area (peer stores
                        // over NVLink; the local one for this rank).
                        for (int q = 0; q < a.tp_world; ++q) a.peer_recv[q][(size_t)a.tp_rank * a.d + row] = sum;
                    } else {
                        if (!waited) {
                            pdl_wait();
                            waited = true;
                        }
                        a.out[(size_t)m * a.d + row] = sum;
                    }
                    if constexpr (EPI == EPI_ARGMAX) {
                        const unsigned long long key = argmax_key(sum, row + a.row_offset);
                        best = key > best ? key : best;
                    }
                }
            }
            if (s + 1 < total) {  // pass this row's running sum to the warp of stage s+1: one tagged word
                const int cn = (c + 1) % NC;
                *reinterpret_cast<volatile unsigned long long *>(&tok[cn * 32 + lane]) =
                    ((unsigned long long)(unsigned)(s + 1) << 32) | (unsigned long long)__float_as_uint(sum);
            }
        }
        if constexpr (EPI == EPI_ARGMAX) {
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(FULL, best, o);
                best = other > best ? other : best;
            }
            if (lane == 0) wkey[c] = best;
        }
    }
    __syncthreads();

    if constexpr (EPI == EPI_PEER) {
        if (tid == 0) {
            // Count this CTA's rows on every rank.  The barrier above orders every thread's peer stores
            // before this thread's system-scope fence, which orders them before the counts: a rank
            // that sees the count sees the rows.  (One fence per CTA: a fence in every thread costs
            // several microseconds per exchange.)
            const int lo = sc.t0 * p.T, hi = min(a.d, (sc.t0 + sc.nt) * p.T);
            const unsigned long long rows = hi > lo ? (unsigned long long)(hi - lo) : 0ull;
            __threadfence_system();
            for (int q = 0; q < a.tp_world; ++q) atomicAdd_system(a.peer_cnt[q], rows);
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (tid == 0) {
            unsigned long long bb = 0ull;
            for (int w = 0; w < NC; ++w) bb = wkey[w] > bb ? wkey[w] : bb;
            a.amax_part[blockIdx.x] = bb;
            __threadfence();
            const unsigned ticket = atomicAdd(a.amax_count, 1u);
            flags[1] = (ticket == gridDim.x - 1);
        }
        __syncthreads();
        if (flags[1] && tid == 0) {
            __threadfence();
            unsigned long long bb = 0ull;
            for (int i = 0; i < (int)gridDim.x; ++i) {
                const unsigned long long kk = __ldcg(a.amax_part + i);
                bb = kk > bb ? kk : bb;
            }
            if (a.tp_world > 1) {
                // Exchange the ranks' best keys (global row indices), then every rank takes the same
                // maximum.
                for (int q = 0; q < a.tp_world; ++q) a.peer_amax[q][a.tp_rank] = bb;
                __threadfence_system();
                for (int q = 0; q < a.tp_world; ++q) atomicAdd_system(a.peer_amax_cnt[q], 1ull);
                wait_counter(a.amax_keys_cnt, (*a.epoch + 1ull) * (unsigned long long)a.tp_world, a.err);
                __threadfence();
                for (int q = 0; q < a.tp_world; ++q) {
                    const unsigned long long k = __ldcg(a.amax_keys + q);
                    bb = k > bb ? k : bb;
                }
                *a.epoch_rw = *a.epoch + 1ull;
            }
            const int vocab = a.vocab > 0 ? a.vocab : a.d;
            int idx = (bb == 0ull) ? 0 : argmax_idx(bb);
            if (idx < 0 || idx >= vocab) idx = 0;
            const int pos = *a.pos;
            if (pos + 1 <= a.seq_len && pos + 1 >= *a.n_forced) a.tokens[pos + 1] = idx;
            *a.pos = pos + 1;
            *a.amax_count = 0u;
        }
    }
}

template <int PRO, int EPI>
cudaError_t launch_t(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl, const GemvBatch &bt = GemvBatch()) {
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
    cfg.gridDim = dim3(p.grid * (bt.count > 0 ? bt.groups : 1));
    cfg.blockDim = dim3(32 * kMinWarps);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, p, bt);
}

}  // namespace

size_t gemv_x_bytes(int n) { return (((size_t)n + 15) & ~(size_t)15) + (size_t)((n / 32 + 3) & ~3) * 4; }

int gemv_tile_rows(int d, int epi, int num_sms) { return q8_tile_rows(d, num_sms, epi == EPI_SWIGLU ? 2 : 1); }

bool gemv_supported(int n, int d, int epi) {
    if (n <= 0 || d <= 0 || n % 32) return false;
    if (epi == EPI_SWIGLU && (d & 1)) return false;
    return gemv_smem_tail(n) + 36 * 1024 < kSmemBudget;  // the activation must fit beside one ring slot
}

size_t gemv_smem_tail(int n) {
    return gemv_x_bytes(n) + kMinWarps * 4 + 2 * kMaxSlots * 8 + kMaxConsumers * 32 * 8 + kMaxConsumers * 8 +
           16;  // activation, red, full/empty, tagged token words, warp keys, flags
}

GemvPlan plan_gemv(int n, int d, int epi, int num_sms) {
    GemvPlan p;
    p.T = gemv_tile_rows(d, epi, num_sms);
    p.ntiles = (d + p.T - 1) / p.T;
    p.grid = std::max(1, std::min(num_sms, p.ntiles));
    const int tiles_per_cta = (p.ntiles + p.grid - 1) / p.grid;
    const int stages = tiles_per_cta * ((n + 511) / 512);
    p.slot = (size_t)p.T * q8_blk_bytes(std::min(n, 512));
    const size_t tail = gemv_smem_tail(n);
    const size_t ring = kSmemBudget > tail ? kSmemBudget - tail : 0;
    // Two producer threads, the deepest ring the budget allows (a multiple of 2), up to 4 consumer
    // warps, and 3 stages of L2 prefetch beyond the ring: the best settings measured on B200 for the
    // LLaMA shapes within the co-residency budget.
    p.NP = 2;
    p.S = std::max(1, std::min({kMaxSlots, (int)(ring / p.slot), stages}));
    if (p.S >= 2) p.S -= p.S % p.NP;
    else p.NP = 1;
    int nc = 4;
    if (const char *e = getenv("DIOLKOS_GEMV_NC")) nc = std::max(1, std::min(atoi(e), kMaxConsumers));
    p.NW = std::max(1, std::min({nc, p.S, stages}));
    p.PF = kPrefetchStages;
    p.xoff = (size_t)p.S * p.slot;
    p.smem = p.xoff + tail;
    return p;
}

GemvPlan plan_gemv_batch(int n, int d, int count, int num_sms) {
    GemvPlan p = plan_gemv(n, d, EPI_STORE, num_sms);
    // the ring as deep as the budget allows: the batch's stages run on from one matrix into the next
    const int stages = ((p.ntiles + p.grid - 1) / p.grid) * ((n + 511) / 512) * std::max(1, count);
    const size_t tail = gemv_smem_tail(n);
    const size_t ring = kSmemBudget > tail ? kSmemBudget - tail : 0;
    p.S = std::max(1, std::min({kMaxSlots, (int)(ring / p.slot), stages}));
    if (p.S >= 2) p.S -= p.S % p.NP;
    int nc = 4;
    if (const char *e = getenv("DIOLKOS_GEMV_NC")) nc = std::max(1, std::min(atoi(e), kMaxConsumers));
    p.NW = std::max(1, std::min({nc, p.S, stages}));
    p.xoff = (size_t)p.S * p.slot;
    p.smem = p.xoff + tail;
    return p;
}

cudaError_t launch_gemv_batch(const GemvArgs &a, const GemvBatch &b, const GemvPlan &p, cudaStream_t st, bool pdl) {
    if (b.count < 1 || b.count > kGemvBatchMax || b.groups < 1 || b.groups > 2 || b.groups > b.count || a.epi != EPI_STORE || (a.pro != PRO_F32 && a.pro != PRO_Q8) ||
        !gemv_supported(a.n, a.d, a.epi) || p.smem > 227 * 1024 || p.NW < 1 || p.NW > kMaxConsumers || p.S < p.NW ||
        p.NP < 1 || p.NW + p.NP > kMinWarps || p.S % p.NP || p.S > kMaxSlots || p.T < 1 || p.T > 32 || p.PF < 0 ||
        p.smem < (size_t)p.S * p.slot + gemv_smem_tail(a.n))
        return cudaErrorInvalidValue;
    for (int i = 0; i < b.count; ++i)
        if (!b.w[i]) return cudaErrorInvalidValue;
    if (a.pro == PRO_Q8) return launch_t<PRO_Q8, EPI_STORE>(a, p, st, pdl, b);
    return launch_t<PRO_F32, EPI_STORE>(a, p, st, pdl, b);
}

cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
    if (!gemv_supported(a.n, a.d, a.epi) || p.smem > 227 * 1024 || p.NW < 1 || p.NW > kMaxConsumers || p.S < p.NW ||
        p.NP < 1 || p.NW + p.NP > kMinWarps || p.S % p.NP ||
        p.S > kMaxSlots || p.T < 1 || p.T > 32 || p.PF < 0 || p.smem < (size_t)p.S * p.slot + gemv_smem_tail(a.n))
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
    DK_GEMV_CASE(PRO_F32, EPI_PEER)
    DK_GEMV_CASE(PRO_RMS_REDUCE, EPI_STORE)
    DK_GEMV_CASE(PRO_RMS_REDUCE, EPI_SWIGLU)
    DK_GEMV_CASE(PRO_RMS_REDUCE, EPI_ARGMAX)
#undef DK_GEMV_CASE
    return cudaErrorInvalidValue;
}

}  // namespace dk
