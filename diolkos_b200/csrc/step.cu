// step.cu -- one whole decode step (reference forward, src/transformer.c:55-239, plus the greedy
// sample_argmax of the generate loop) as ONE persistent kernel on sm_100a.
//
// Grid: one CTA per SM, launched cooperatively (all CTAs resident).  The step is a list of OPS built
// on the host: per layer a q|k|v GEMV, attention, wo GEMV, w1|w3 GEMV and w2 GEMV, then the
// classifier GEMV.  Every CTA walks the list in order.
//
//  * Two PRODUCER warps (one thread each) stream every GEMV stage this CTA owns -- in op order, ACROSS
//    op boundaries -- through a ring of S shared-memory slots with the bulk-copy engine.  Weights never
//    depend on activations, so while the CTA waits for an op's input (or runs attention) the ring keeps
//    filling with the next matrix: the HBM stream does not stop between matrices the way it does
//    between separate kernels.
//  * Ten COMPUTE warps.  For a GEMV op: wait until the op's input is complete, build the Q8_0
//    activation in shared memory (rmsnorm, embedding-row dequant or the tensor-parallel reduce fused
//    in), then NC of them consume the stages exactly as the standalone GEMV does (gemv_core.cuh: the
//    same bit-exact terms and in-order row sums), and the epilogue stores the rows.  For attention:
//    five groups of two warps take (KV head, position split) items, flash-decoding style, and the last
//    split of a head merges.
//  * Dependencies between ops are COUNTERS in global memory, not grid barriers: an op adds the units
//    it completed (rows, attention outputs) after a release fence, and a consumer op waits (bounded,
//    acquire) until the counter reaches (epoch + 1) * units.  epoch = decode steps completed; the
//    classifier's last CTA advances it, so counters never need resetting.  A CTA that owns no rows of
//    an op neither reads its input nor counts, so every reader of a buffer has counted before anyone
//    can overwrite it (the dataflow chain of the step orders all reuse).  The residual a prologue
//    produces (embedding row, tensor-parallel sum) is stored by the CTA that owns the op's tile 0.
//
// Tensor parallel: wo / w2 store their partial rows into every rank's receive area (EPI_PEER) and the
// next GEMV's prologue waits for all ranks' rows (PRO_RMS_REDUCE), exactly as the standalone kernels
// do; only the waiting moved into the persistent kernel, where the weight stream hides it.
//
// Every wait is bounded (DK_WAIT_LIMIT_CYCLES): on a timeout the waiter records the error word and
// raises the CTA's abort flag; all warps leave their loops at the next check, and the producers wait
// for their copies in flight before the CTA exits.
#include "dk_common.cuh"
#include "dk_kernels.h"
#include "gemv_core.cuh"

#include <algorithm>
#include <cstdio>

namespace dk {
namespace {

constexpr int kStepWarps = 12;
constexpr int kStepThreads = 32 * kStepWarps;
constexpr int kComputeWarps = kStepWarps - kStepProducers;  // warps 0 .. 9
constexpr int kComputeThreads = 32 * kComputeWarps;
// Attention items run on groups of GW warps: kAttnNarrowWarps (the narrow form: kComputeWarps / GW groups
// per CTA) or kAttnWideWarps (the wide form: one group, every compute warp), step_attn_plan.
constexpr int kAttnGroups = kComputeWarps / kAttnNarrowWarps;  // groups of the narrow form (5)
static_assert(kAttnWideWarps == kComputeWarps && kComputeWarps % kAttnNarrowWarps == 0, "attention groups");
constexpr int kBatch = 8;          // positions an attention warp loads at once
constexpr int kHeadsPerPass = 2;   // query heads of one KV head an attention warp holds at once
constexpr int kMergeChunk = 12;    // splits whose partials the merging group loads in one round trip
// head dims per merging thread of a GW-warp group (head_size <= 128)
template <int GW> constexpr int merge_dims() { return (128 + 32 * GW - 1) / (32 * GW); }
constexpr int kBarCompute = 1;     // named barrier of the compute warps; 2 + g: attention group g
constexpr int kStepActBlocks = 64; // 512-column blocks of an activation built block by block (n <= 32768)
static_assert(2 + kAttnGroups <= 16, "named barriers");

struct StepCtl {  // shared-memory control block
    uint64_t full[kStepMaxSlots];    // ring slot holds its stage's weights
    uint64_t empty[kStepMaxSlots];   // ring slot read by its consumer
    unsigned long long wkey[kStepMaxConsumers];  // consumers' best greedy-token keys of the op
    float red[kStepWarps];
    // running row sums handed to each consumer warp, one 64-bit word per lane: the global index of the
    // stage they are for (high half) and the sum's bits (low half), stored and polled as one word
    unsigned long long tok[kStepMaxConsumers][32];
    int abort;      // any wait gave up: every warp leaves
    int last;       // this CTA took the classifier's last ticket
    int crit;       // the compute warps wait for an op's input, build its activation or run attention
    int grp_last[kAttnGroups];
    // per 512-column block of a PRO_F32 op's activation: the op index + 1 once its values and scales are in
    // shared memory (step_activation_blocks)
    int act_ready[kStepActBlocks];
    // The compute warps' copies of the op descriptors: op i sits in opbuf[i % 3].  Op i+1 is loaded into
    // registers while op i runs and stored here before op i's last barrier, so no read of a descriptor
    // waits on the L2 at an op boundary; three slots keep op i-1's descriptor intact for its stragglers.
    alignas(16) unsigned long long opbuf[3][(sizeof(StepOp) + 7) / 8];
};
constexpr int kOpWords = (int)((sizeof(StepOp) + 7) / 8);
static_assert(kOpWords <= kComputeThreads - 32, "one descriptor word per thread of warps 1..");

// Self-checking build (-DDK_STEP_CHECKS): every global and shared access below whose index is not
// trivially in range is tested first; a failed test records the site and value (first one only, with
// a device printf), raises DK_ERR_INVALID and skips the access.  Off in normal builds.
#ifdef DK_STEP_CHECKS
__device__ __forceinline__ bool step_chk(bool ok, int *err, int site, long long v) {
    if (!ok) {
        if (atomicCAS(err + 1, 0, site) == 0)
            printf("step check failed: site %d value %lld block %d thread %d\n", site, v, (int)blockIdx.x, (int)threadIdx.x);
        atomicOr(err, DK_ERR_INVALID);
    }
    return ok;
}
#define DK_CHK(cond, err, site, v) step_chk((cond), (err), (site), (long long)(v))
#else
#define DK_CHK(cond, err, site, v) true
#endif

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Optional timeline (StepArgs::trace): per CTA and op, [0] input ready (after the CTA barrier),
// [1] activation built, [2] op finished on this CTA, [3] the producers' last stage of the op issued,
// [4] the input counter seen by the polling thread.
constexpr int kTraceSlots = 8;
__device__ __forceinline__ void trace_mark(const StepArgs &sa, int op, int k) {
    if (sa.trace) sa.trace[((size_t)blockIdx.x * sa.nops + op) * kTraceSlots + k] = globaltimer();
}

__device__ __forceinline__ void bar_compute() {
    asm volatile("bar.sync %0, %1;" ::"n"(kBarCompute), "n"(kComputeThreads) : "memory");
}
// The compute warps' barrier that also tells every thread whether any of them passed v != 0: a flag
// that another warp may raise while the compute warps arrive (the producers' abort) is read once per
// thread before the barrier, and the OR makes the decision to leave the op loop the same everywhere.
__device__ __forceinline__ bool bar_compute_or(int v) {
    unsigned r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(v), "n"(kBarCompute), "n"(kComputeThreads)
        : "memory");
    return r != 0;
}
template <int GW>
__device__ __forceinline__ void bar_group(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(2 + g), "n"(32 * GW) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Add to a completion counter with release semantics: the calling thread's CTA barrier has ordered the
// CTA's stores before it, and the release makes them visible to whoever acquires the new count.
__device__ __forceinline__ void red_release_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded wait until a counter of this GPU reaches target.
__device__ __forceinline__ bool wait_local(const unsigned long long *cnt, unsigned long long target, int *err) {
    if (ld_acquire_gpu(cnt) >= target) return true;
    const long long t0 = clock64();
    while (ld_acquire_gpu(cnt) < target) {
        if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
            atomicOr(err, DK_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// The CTA's stages of a GEMV op: tile t0 + s / nblk, block s % nblk, for s < nst.
__device__ __forceinline__ Sched op_sched(const StepOp &op) {
    Sched sc;
    sc.t0 = (int)((long long)blockIdx.x * op.ntiles / gridDim.x);
    sc.nt = (int)((long long)(blockIdx.x + 1) * op.ntiles / gridDim.x) - sc.t0;
    sc.nblk = (op.g.n + 511) >> 9;
    sc.T = op.T;
    sc.n = op.g.n;
    sc.nst = sc.nt * sc.nblk;
    sc.tile_bytes = (size_t)op.T * q8_row_bytes(op.g.n);
    return sc;
}

__device__ __forceinline__ size_t gemv_x_bytes_dev(int n) {
    return (((size_t)n + 15) & ~(size_t)15) + (size_t)((n / 32 + 3) & ~3) * 4;
}

// ---- tensor parallel: the tagged exchange (GemvArgs::tagged) ------------------------------------------
__device__ __forceinline__ unsigned tp_tag(unsigned long long epoch, const GemvArgs &a, int k) {
    return (unsigned)(epoch * (unsigned long long)a.tag_period + (unsigned long long)(k + 1));
}
__device__ __forceinline__ void ld_v2u64(const unsigned long long *p, unsigned long long &x, unsigned long long &y) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
}
__device__ __forceinline__ void st_v2u64(unsigned long long *p, unsigned long long x, unsigned long long y) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y) : "memory");
}
__device__ __forceinline__ void st_u64(unsigned long long *p, unsigned long long x) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(x) : "memory");
}
__device__ __forceinline__ unsigned long long tagged_word(unsigned T, float v) {
    return ((unsigned long long)T << 32) | (unsigned long long)__float_as_uint(v);
}
// Wait (bounded) until the N words at p (16-byte aligned) all carry tag T, and take their values.  A word
// is single-copy atomic, so a value arrives with its tag whether a peer GPU or another CTA wrote it.  On a
// timeout: DK_ERR_COMM, zeros, false -- the caller carries on through its barriers and aborts after them.
template <int N>
__device__ __forceinline__ bool wait_tagged(const unsigned long long *p, unsigned T, float (&v)[N], int *err) {
    static_assert(N % 2 == 0, "pairs of words");
    unsigned long long w[N];
    const long long t0 = clock64();
    for (;;) {
        #pragma unroll
        for (int i = 0; i < N; i += 2) ld_v2u64(p + i, w[i], w[i + 1]);
        bool ok = true;
        #pragma unroll
        for (int i = 0; i < N; ++i) ok &= (unsigned)(w[i] >> 32) == T;
        if (ok) {
            #pragma unroll
            for (int i = 0; i < N; ++i) v[i] = __uint_as_float((unsigned)w[i]);
            return true;
        }
        if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
            atomicOr(err, DK_ERR_COMM);
            #pragma unroll
            for (int i = 0; i < N; ++i) v[i] = 0.0f;
            return false;
        }
    }
}
// Gatherer CTA (blockIdx.x < n_gather) of a reduce: for its slice of the rows, every rank's partial sum
// (event tag_k) added in rank order onto the residual (event tag_k - 1), x + (p_0 + p_1 + ...) as the
// counter exchange computes it, published as the new tagged residual.
__device__ bool tp_gather(const GemvArgs &a, unsigned long long epoch, int tid) {
    const int n = a.n, NG = a.n_gather;
    const int per = ((n + NG - 1) / NG + 3) & ~3;
    const int r0 = (int)blockIdx.x * per, r1 = min(n, r0 + per);
    const unsigned T = tp_tag(epoch, a, a.tag_k), Tx = tp_tag(epoch, a, a.tag_k - 1);
    bool ok = true;
    for (int r = r0 + 4 * tid; r + 4 <= r1; r += 4 * kComputeThreads) {
        float x[4], t[4], u[4];
        ok &= wait_tagged<4>(a.x64 + r, Tx, x, a.err);
        ok &= wait_tagged<4>(a.recv64 + r, T, t, a.err);
        for (int q = 1; q < a.tp_world; ++q) {
            ok &= wait_tagged<4>(a.recv64 + (size_t)q * n + r, T, u, a.err);
            #pragma unroll
            for (int j = 0; j < 4; ++j) t[j] = __fadd_rn(t[j], u[j]);
        }
        st_v2u64(a.x64_out + r, tagged_word(T, __fadd_rn(x[0], t[0])), tagged_word(T, __fadd_rn(x[1], t[1])));
        st_v2u64(a.x64_out + r + 2, tagged_word(T, __fadd_rn(x[2], t[2])), tagged_word(T, __fadd_rn(x[3], t[3])));
    }
    return ok;
}

// ---- activation prologue (compute threads) ------------------------------------------------------
// 16 consecutive values of the op's input, half-group hg (values 16hg .. 16hg+15).  The tagged reduce reads
// the new residual its gatherers published (tag T; ok = false on a timeout).
__device__ __forceinline__ void load16(const GemvArgs &a, int tok, int hg, float (&f)[16], unsigned T, bool &ok) {
    const int n = a.n;
    if (a.pro == PRO_RMS_REDUCE && a.tagged) {
        ok &= wait_tagged<16>(a.x64_out + 16 * hg, T, f, a.err);
        return;
    }
    if (a.pro == PRO_EMB_RMS) {
        if (!DK_CHK(tok >= 0 && tok < (a.vocab > 0 ? a.vocab : 1) && hg < (n >> 4), a.err, 10, tok)) {
            #pragma unroll
            for (int i = 0; i < 16; ++i) f[i] = 0.0f;
            return;
        }
        // the embedding row's group g = hg/2, half hg&1 (src/transformer.c:69)
        const int g = hg >> 1, b = g >> 4, wb = q8_blk_width(n, b), r = tok % a.emb_T, k = g & 15;
        const uint8_t *seg = a.emb + q8_seg_off(n, a.emb_T, tok, b);
        const uint4 c = __ldg(reinterpret_cast<const uint4 *>(seg + 16 * q8_swz_q(2 * k + (hg & 1), r, wb)));
        const float s = __ldg(reinterpret_cast<const float *>(seg + wb + 16 * q8_swz_s(k >> 2, r, wb) + 4 * (k & 3)));
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        #pragma unroll
        for (int i = 0; i < 16; ++i) f[i] = __fmul_rn((float)(int8_t)(w[i >> 2] >> (8 * (i & 3))), s);
        return;
    }
    float4 v[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = __ldcg(reinterpret_cast<const float4 *>(a.x + 16 * hg) + k);
    if (a.pro == PRO_RMS_REDUCE) {
        // x + (partial_0 + partial_1 + ...), ranks in order: the same bits on every rank
        float4 t[4];
        #pragma unroll
        for (int k = 0; k < 4; ++k) t[k] = __ldcg(reinterpret_cast<const float4 *>(a.recv + 16 * hg) + k);
        for (int q = 1; q < a.tp_world; ++q) {
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 u = __ldcg(reinterpret_cast<const float4 *>(a.recv + (size_t)q * n + 16 * hg) + k);
                t[k] = make_float4(__fadd_rn(t[k].x, u.x), __fadd_rn(t[k].y, u.y), __fadd_rn(t[k].z, u.z),
                                   __fadd_rn(t[k].w, u.w));
            }
        }
        #pragma unroll
        for (int k = 0; k < 4; ++k)
            v[k] = make_float4(__fadd_rn(v[k].x, t[k].x), __fadd_rn(v[k].y, t[k].y), __fadd_rn(v[k].z, t[k].z),
                               __fadd_rn(v[k].w, t[k].w));
    }
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
        f[4 * k] = v[k].x; f[4 * k + 1] = v[k].y; f[4 * k + 2] = v[k].z; f[4 * k + 3] = v[k].w;
    }
}

// Quantise 16 values (one half of a group; the partner half is the neighbouring lane) into xq/xs.
__device__ __forceinline__ void quant16(float (&f)[16], int hg, bool live, int8_t *xq, float *xs) {
    float amax = 0.0f;
    #pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(f[k]));
    amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 1));  // the group's other half
    float sc, inv;
    q8_scale(amax, sc, inv);
    if (!live) return;
    uint32_t wq[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k)
        wq[k] = (uint32_t)(uint8_t)q8_round(f[4 * k], inv) | ((uint32_t)(uint8_t)q8_round(f[4 * k + 1], inv) << 8) |
                ((uint32_t)(uint8_t)q8_round(f[4 * k + 2], inv) << 16) |
                ((uint32_t)(uint8_t)q8_round(f[4 * k + 3], inv) << 24);
    reinterpret_cast<uint4 *>(xq + 16 * hg)[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
    if (!(hg & 1)) xs[hg >> 1] = sc;
}

// Build the op's Q8_0 activation (xq int8[n], xs fp32[n/32]) with the compute threads.  Thread t
// takes half-groups t, t + 320, ...; the rmsnorm family keeps up to two rounds in registers.
// Returns false if a wait gave up.
// writer: this CTA owns tile 0 of the op, so it stores the residual the prologue produces (the
// embedding row, or x plus the ranks' partials): exactly one CTA of the grid does.
// nw0: this thread's norm weights for round 0 (loaded before the input wait: they are constant).
__device__ bool step_activation(const GemvArgs &a, int tok, int8_t *xq, float *xs, StepCtl &ctl, int tid,
                                unsigned long long epoch, bool writer, const float4 (&nw0)[4]) {
    const int n = a.n, nhg = n >> 4, warp = tid >> 5, lane = tid & 31;
    bool ok = true;  // false: a tagged wait gave up (every barrier below is still taken)
    const unsigned T = a.tagged ? tp_tag(epoch, a, a.tag_k) : 0u;
    if (a.pro == PRO_RMS_REDUCE && !a.tagged) {
        // every rank's partial rows for this exchange point have landed once the counter reaches this
        if (tid == 0) {
            const unsigned long long target =
                (epoch * (unsigned long long)a.red_period + (unsigned long long)a.red_index + 1ull) *
                (unsigned long long)a.tp_world * (unsigned long long)n;
            if (!wait_counter(a.cnt, target, a.err)) ctl.abort = 1;
        }
        if (bar_compute_or(*reinterpret_cast<volatile int *>(&ctl.abort))) return false;  // the same for every thread
        __threadfence();
    }
    const bool rms = a.pro == PRO_RMS || a.pro == PRO_EMB_RMS || a.pro == PRO_RMS_REDUCE;
    // the residual the prologue produces, stored by one CTA: the embedding row (tagged under the tagged
    // exchange), or the untagged reduce's sum (the tagged reduce's gatherers stored theirs)
    const bool write_x = writer && (a.pro == PRO_EMB_RMS || (a.pro == PRO_RMS_REDUCE && !a.tagged));
    const bool write_x64 = write_x && a.tagged;
    float *xdst = a.pro == PRO_RMS_REDUCE ? a.x_out : const_cast<float *>(a.x);
    const int rounds = (nhg + kComputeThreads - 1) / kComputeThreads;
    if (rms && rounds <= 2) {
        float f0[16], f1[16];
        float ss = 0.0f;
        #pragma unroll
        for (int k = 0; k < 2; ++k) {
            float(&f)[16] = k == 0 ? f0 : f1;
            const int hg = k * kComputeThreads + tid;
            const bool live = k < rounds && hg < nhg;
            if (live) {
                load16(a, tok, hg, f, T, ok);
                if (write_x64) {
                    #pragma unroll
                    for (int j = 0; j < 16; j += 2)
                        st_v2u64(a.x64_out + 16 * hg + j, tagged_word(T, f[j]), tagged_word(T, f[j + 1]));
                } else if (write_x) {
                    #pragma unroll
                    for (int j = 0; j < 4; ++j)
                        reinterpret_cast<float4 *>(xdst + 16 * hg)[j] =
                            make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
                }
                #pragma unroll
                for (int j = 0; j < 16; ++j) ss = fmaf(f[j], f[j], ss);
            } else {
                #pragma unroll
                for (int j = 0; j < 16; ++j) f[j] = 0.0f;
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) ctl.red[warp] = ss;
        bar_compute();
        float tot = 0.0f;
        #pragma unroll
        for (int w = 0; w < kComputeWarps; ++w) tot += ctl.red[w];
        // rmsnorm (src/utils.c:68-75): 1/sqrt(ss/n + 1e-5), o = (w*x)*scale
        float r = __fdiv_rn(tot, (float)n);
        r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(r, 1e-5f)));
        #pragma unroll
        for (int k = 0; k < 2; ++k) {
            float(&f)[16] = k == 0 ? f0 : f1;
            const int hg = k * kComputeThreads + tid;
            if (k >= rounds) break;  // uniform
            const bool live = hg < nhg;
            if (live) {
                #pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 w = k == 0 ? nw0[j] : __ldg(reinterpret_cast<const float4 *>(a.norm_w + 16 * hg) + j);
                    f[4 * j] = __fmul_rn(__fmul_rn(w.x, f[4 * j]), r);
                    f[4 * j + 1] = __fmul_rn(__fmul_rn(w.y, f[4 * j + 1]), r);
                    f[4 * j + 2] = __fmul_rn(__fmul_rn(w.z, f[4 * j + 2]), r);
                    f[4 * j + 3] = __fmul_rn(__fmul_rn(w.w, f[4 * j + 3]), r);
                }
            }
            quant16(f, hg, live, xq, xs);
        }
        return ok;
    }
    if (!rms && rounds <= 3) {
        // plain quantisation of up to three rounds: every load is issued before any is used
        float f[3][16];
        #pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int hg = k * kComputeThreads + tid;
            if (k < rounds && hg < nhg) {
                load16(a, tok, hg, f[k], T, ok);
            } else {
                #pragma unroll
                for (int j = 0; j < 16; ++j) f[k][j] = 0.0f;
            }
        }
        #pragma unroll
        for (int k = 0; k < 3; ++k) {
            if (k >= rounds) break;  // uniform
            const int hg = k * kComputeThreads + tid;
            quant16(f[k], hg, hg < nhg, xq, xs);
        }
        return ok;
    }
    float r = 1.0f;
    if (rms) {  // wide rmsnorm input: sum of squares first, values re-read below
        float ss = 0.0f;
        for (int hg = tid; hg < nhg; hg += kComputeThreads) {
            float f[16];
            load16(a, tok, hg, f, T, ok);
            if (write_x64) {
                #pragma unroll
                for (int j = 0; j < 16; j += 2)
                    st_v2u64(a.x64_out + 16 * hg + j, tagged_word(T, f[j]), tagged_word(T, f[j + 1]));
            } else if (write_x) {
                #pragma unroll
                for (int j = 0; j < 4; ++j)
                    reinterpret_cast<float4 *>(xdst + 16 * hg)[j] = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
            }
            #pragma unroll
            for (int j = 0; j < 16; ++j) ss = fmaf(f[j], f[j], ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) ctl.red[warp] = ss;
        bar_compute();
        float tot = 0.0f;
        #pragma unroll
        for (int w = 0; w < kComputeWarps; ++w) tot += ctl.red[w];
        r = __fdiv_rn(tot, (float)n);
        r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(r, 1e-5f)));
    }
    for (int base = 0; base < nhg; base += kComputeThreads) {  // uniform trip count: shuffles stay full-warp
        const int hg = base + tid;
        const bool live = hg < nhg;
        float f[16];
        if (live) {
            load16(a, tok, hg, f, T, ok);
            if (rms) {
                #pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 w = __ldg(reinterpret_cast<const float4 *>(a.norm_w + 16 * hg) + j);
                    f[4 * j] = __fmul_rn(__fmul_rn(w.x, f[4 * j]), r);
                    f[4 * j + 1] = __fmul_rn(__fmul_rn(w.y, f[4 * j + 1]), r);
                    f[4 * j + 2] = __fmul_rn(__fmul_rn(w.z, f[4 * j + 2]), r);
                    f[4 * j + 3] = __fmul_rn(__fmul_rn(w.w, f[4 * j + 3]), r);
                }
            }
        } else {
            #pragma unroll
            for (int j = 0; j < 16; ++j) f[j] = 0.0f;
        }
        quant16(f, hg, live, xq, xs);
    }
    return ok;
}

// The Q8_0 activation of a PRO_F32 op (a plain per-group quantisation, no norm: wo on the attention
// output, w2 on the SwiGLU output) built block by block by the compute warps that do not consume, in
// block order (builder k of NB takes blocks k, k + NB, ...), each block published with act_ready[b] =
// tag.  The consumers start on block 0 as soon as it is there instead of waiting for the whole vector.
// The arithmetic is step_activation's (load16 / quant16): the same bits.
__device__ void step_activation_blocks(const GemvArgs &a, int8_t *xq, float *xs, StepCtl &ctl, int k, int NB,
                                       int lane, int tag) {
    const int nhg = a.n >> 4, nblk = (a.n + 511) >> 9;
    bool ok = true;
    for (int b = k; b < nblk; b += NB) {
        const int hg = 32 * b + lane;  // half-group: 16 values; the partner half is the neighbouring lane
        float f[16];
        if (hg < nhg) {
            load16(a, 0, hg, f, 0u, ok);
        } else {
            #pragma unroll
            for (int j = 0; j < 16; ++j) f[j] = 0.0f;
        }
        quant16(f, hg, hg < nhg, xq, xs);
        __threadfence_block();  // this lane's values and scale before the block's flag
        __syncwarp();
        if (lane == 0)
            asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(&ctl.act_ready[b])), "r"(tag)
                         : "memory");
    }
}
// Bounded wait (acquire) until block b of the activation is published; abandoned on the abort flag.
__device__ __forceinline__ bool wait_act_block(const StepCtl &ctl, int b, int tag, int *err, const int *abort) {
    const uint32_t w = smem_u32(&ctl.act_ready[b]);
    int v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(w) : "memory");
    if (v == tag) return true;
    const long long t0 = clock64();
    for (int it = 1;; ++it) {
        asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(w) : "memory");
        if (v == tag) return true;
        if (!(it & 15)) {
            if (*reinterpret_cast<const volatile int *>(abort)) return false;
            if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
                atomicOr(err, DK_ERR_TIMEOUT);
                return false;
            }
        }
    }
}

// ---- GEMV op: consumers ---------------------------------------------------------------------------
// Consume this CTA's stages of the op (compute warp c < NC): the standalone GEMV's arithmetic
// (gemv_core.cuh) with the ring position continuing from `gbase` (stages of earlier ops).  The stages
// are taken in UNITS of two consecutive blocks of one tile (one block where a tile has an odd count):
// unit u goes to warp u % NC, which computes both stages' group terms, frees their ring slots, and then
// waits for the rows' running sums after unit u-1 (the TOKEN, flagged with the global index of the
// unit's first stage), adds its 32 terms in group order, and passes the sums on.  So every row is
// summed in the reference's group order while the terms of NC units are computed at once, and the
// sums cross between warps once per two blocks.  Returns false on abort.

// The terms of stage G (block b of the tile whose row this lane owns) into t, then its slot freed.
__device__ __forceinline__ bool stage_terms(const GemvArgs &a, int G, int b, int S, size_t slot_bytes, uint32_t ring_s,
                                            uint32_t xq_s, uint32_t xs_s, StepCtl &ctl, int lane, bool live,
                                            float (&t)[16], unsigned long long *st, int act_tag) {
    const int slot = G % S;
    if (!__all_sync(FULL, mbar_wait_abortable(&ctl.full[slot], (uint32_t)((G / S) & 1), a.err, &ctl.abort, false) &&
                              (act_tag == 0 || wait_act_block(ctl, b, act_tag, a.err, &ctl.abort)))) {
        if (lane == 0) ctl.abort = 1;
        return false;
    }
    if (st) st[0] = globaltimer();
    const int wb = q8_blk_width(a.n, b);
    if (live && DK_CHK((size_t)slot * slot_bytes + (size_t)(lane + 1) * q8_blk_bytes(wb) <= (size_t)S * slot_bytes &&
                           512 * b + wb <= a.n,
                       a.err, 2, G)) {
        const uint32_t seg = ring_s + (uint32_t)(slot * slot_bytes + lane * q8_blk_bytes(wb));
        const uint32_t xqb = xq_s + 512u * b, xsb = xs_s + 64u * b;
        if (wb == 512) block_terms_full(t, seg, xqb, xsb, lane);
        else block_terms_part(t, seg, xqb, xsb, wb, lane);
        // pinned here: otherwise the compiler may sink the term arithmetic past the token wait
        #pragma unroll
        for (int g = 0; g < 16; ++g) asm volatile("" : "+f"(t[g]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl.empty[slot]);
    if (st) st[1] = globaltimer();
    return true;
}
__device__ __forceinline__ float add_terms(float sum, const float (&t)[16], int wb) {
    if (wb == 512) {
        #pragma unroll
        for (int g = 0; g < 16; ++g) sum = __fadd_rn(sum, t[g]);
    } else {
        #pragma unroll
        for (int g = 0; g < 16; ++g)
            if (g < (wb >> 5)) sum = __fadd_rn(sum, t[g]);
    }
    return sum;
}

__device__ bool gemv_consume(const StepOp &op, const Sched &sc, int gbase, int S, int NC, size_t slot_bytes,
                             uint32_t ring_s, uint32_t xq_s, uint32_t xs_s, StepCtl &ctl, int c, int lane,
                             unsigned long long &best, unsigned long long *strace, unsigned long long epoch,
                             int act_tag) {
    const GemvArgs &a = op.g;
    const int n = a.n;
    const unsigned T = a.tagged ? tp_tag(epoch, a, a.tag_k) : 0u;
    const int upt = (sc.nblk + 1) >> 1;  // units per tile
    const int nunits = sc.nt * upt;
    for (int u = c; u < nunits; u += NC) {
        const int tile = u / upt, b0 = 2 * (u - tile * upt);
        const bool two = b0 + 1 < sc.nblk;
        const int s0 = tile * sc.nblk + b0, G0 = gbase + s0;
        const int row = (sc.t0 + tile) * op.T + lane;
        const bool live = lane < op.T && row < a.d;
        unsigned long long *st0 = (strace && s0 < kStageTraceStages && lane == 0) ? strace + 4 * s0 : nullptr;
        unsigned long long *st1 = (strace && s0 + 1 < kStageTraceStages && lane == 0 && two) ? strace + 4 * (s0 + 1) : nullptr;
        const bool last = b0 + (two ? 1 : 0) == sc.nblk - 1;  // this unit finishes the tile's rows
        // the residual the rows add to, loaded before the terms: it is constant during the op (the
        // previous residual add completed before this op's input did), and its L2 round trip would
        // otherwise sit on the tile's last hand-off
        const float res = (last && a.epi == EPI_ADD && live) ? __ldcg(a.out + row) : 0.0f;
        float t0[16] = {}, t1[16] = {};
        if (!stage_terms(a, G0, b0, S, slot_bytes, ring_s, xq_s, xs_s, ctl, lane, live, t0, st0, act_tag)) return false;
        if (two && !stage_terms(a, G0 + 1, b0 + 1, S, slot_bytes, ring_s, xq_s, xs_s, ctl, lane, live, t1, st1, act_tag))
            return false;
        float sum = 0.0f;
        if (u > 0) {  // the running sum of this lane's row after unit u-1
            float prev = 0.0f;
            if (!__all_sync(FULL, lane_token_wait(ctl.tok[c], lane, G0, prev, a.err, &ctl.abort))) {
                if (lane == 0) ctl.abort = 1;
                return false;
            }
            if (b0 > 0) sum = prev;
        }
        if (st0) st0[2] = globaltimer();
        if (live) {
            sum = add_terms(sum, t0, q8_blk_width(n, b0));
            if (two) sum = add_terms(sum, t1, q8_blk_width(n, b0 + 1));
        }
        if (last) {  // the tile's rows are finished
            if (a.epi == EPI_SWIGLU) {
                const float h3 = __shfl_down_sync(FULL, sum, 1);
                if (live && !(lane & 1) && DK_CHK((row >> 1) < (a.d >> 1), a.err, 4, row)) {
                    // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                    float v = __fmul_rn(sum, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-sum))));
                    a.out[row >> 1] = __fmul_rn(v, h3);
                }
            } else if (live) {
                if (a.epi == EPI_ADD) {
                    a.out[row] = __fadd_rn(res, sum);
                } else if (a.epi == EPI_PEER) {
                    if (a.tagged) {  // one tagged word per rank: its own validity, no fence, no count
                        const unsigned long long wv = tagged_word(T, sum);
                        for (int q = 0; q < a.tp_world; ++q) st_u64(a.peer_recv64[q] + (size_t)a.tp_rank * a.d + row, wv);
                    } else {
                        for (int q = 0; q < a.tp_world; ++q) a.peer_recv[q][(size_t)a.tp_rank * a.d + row] = sum;
                    }
                } else {
                    a.out[row] = sum;
                }
                if (a.epi == EPI_ARGMAX) {
                    const unsigned long long key = argmax_key(sum, row + a.row_offset);
                    best = key > best ? key : best;
                }
            }
        }
        if (u + 1 < nunits) {  // hand this row's running sum to the warp of unit u+1: one tagged word
            const int cn = (c + 1) % NC;
            *reinterpret_cast<volatile unsigned long long *>(&ctl.tok[cn][lane]) =
                ((unsigned long long)(unsigned)(G0 + (two ? 2 : 1)) << 32) | (unsigned long long)__float_as_uint(sum);
        }
        if (st0) st0[3] = globaltimer();
    }
    return true;
}

// ---- attention op ----------------------------------------------------------------------------------
template <bool F32>
__device__ __forceinline__ float4 load_kv4(const void *base, size_t idx) {
    if constexpr (F32) {
        return __ldcg(reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx));
    } else {
        const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + idx));
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
// RoPE (src/transformer.c:87-119, HF rotate-half) of dims d0..d0+3 of head vector v, as the reference's
// compiled code evaluates it: a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c).
__device__ __forceinline__ float4 rope4(const float *v, const float *cs, int d0, int half) {
    float r[4];
    #pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int d = d0 + e;
        if (d < half) {
            const float c = __ldg(cs + 2 * d), sn = __ldg(cs + 2 * d + 1);
            r[e] = __fmaf_rn(__ldcg(v + d), c, -__fmul_rn(__ldcg(v + d + half), sn));
        } else {
            const int j = d - half;
            const float c = __ldg(cs + 2 * j), sn = __ldg(cs + 2 * j + 1);
            r[e] = __fmaf_rn(__ldcg(v + j), sn, __fmul_rn(__ldcg(v + d), c));
        }
    }
    return make_float4(r[0], r[1], r[2], r[3]);
}
__device__ __forceinline__ float dot4(float4 a, float4 b) {
    return __fmaf_rn(a.w, b.w, __fmaf_rn(a.z, b.z, __fmaf_rn(a.y, b.y, __fmul_rn(a.x, b.x))));
}

// K and V rows tb .. tb+kBatch-1 of this lane's 4 dims (row pos comes from registers: this step's k, v).
template <bool F32>
__device__ __forceinline__ void load_kv_batch(const AttnArgs &a, size_t head_base, int hs, int tb, int t1, int pos,
                                              bool act, float4 kp, float4 vp, float4 (&kk)[kBatch],
                                              float4 (&vv)[kBatch]) {
    #pragma unroll
    for (int j = 0; j < kBatch; ++j) {
        const int t = tb + j;
        if (t < t1 && act && t != pos) {
            kk[j] = load_kv4<F32>(a.k_cache, head_base + (size_t)t * hs);
            vv[j] = load_kv4<F32>(a.v_cache, head_base + (size_t)t * hs);
        } else {
            kk[j] = (t == pos) ? kp : make_float4(0, 0, 0, 0);
            vv[j] = (t == pos) ? vp : make_float4(0, 0, 0, 0);
        }
    }
}

// One (KV head, split) item on attention group grp (GW warps): the arithmetic of the standalone attention
// kernel (attention.cu), with the group's named barrier in place of the CTA's.  sm = the group's scratch
// [GW][kv_mul][hs + 4].  The output of a KV head's query heads is complete when its last split has
// merged; that split counts them on done_cnt.
template <bool F32, int GW>
__device__ void attn_item(const AttnArgs &a, int pos, int kvh, int split, int nsplit, int chunk, int grp, int gt,
                          float *sm, StepCtl &ctl, unsigned long long *done_cnt, const StepArgs &sa, int opi) {
    const bool mark = grp == 0 && gt == 0 && sa.trace;
    const int lane = gt & 31, warp = gt >> 5;
    const int hs = a.head_size, half = hs >> 1;
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const int dim = a.n_heads * hs, kv_dim = a.n_kv_heads * hs;
    const int t0 = split * chunk, t1 = min(pos + 1, t0 + chunk);
    const int d0 = 4 * lane;
    const bool act = d0 < hs;
    const float *cs = a.rope + (size_t)pos * hs;
    const size_t head_base = (size_t)kvh * a.seq_len * hs + d0;
    if (!DK_CHK(kvh < a.n_kv_heads && split < a.max_splits && pos < a.seq_len && t0 <= pos && kv_mul <= 8 &&
                    (size_t)(kvh + 1) * a.seq_len * hs <= (size_t)a.n_kv_heads * a.seq_len * hs,
                a.err, 5, kvh * 1000 + split))
        return;

    float4 kp = make_float4(0, 0, 0, 0), vp = kp;
    if (pos >= t0 && pos < t1 && act) {
        const float4 kr = rope4(a.qkv + dim + (size_t)kvh * hs, cs, d0, half);
        const float4 vr = __ldcg(reinterpret_cast<const float4 *>(a.qkv + dim + kv_dim + (size_t)kvh * hs + d0));
        kp = make_float4(round_kv<F32>(kr.x), round_kv<F32>(kr.y), round_kv<F32>(kr.z), round_kv<F32>(kr.w));
        vp = make_float4(round_kv<F32>(vr.x), round_kv<F32>(vr.y), round_kv<F32>(vr.z), round_kv<F32>(vr.w));
        if (warp == 0) {
            store_kv4<F32>(a.k_cache, head_base + (size_t)pos * hs, kr);
            store_kv4<F32>(a.v_cache, head_base + (size_t)pos * hs, vr);
        }
    }
    const float sq = __fsqrt_rn((float)hs);
    const int SW = hs + 4;
    // Query heads in passes of kHeadsPerPass (bounded registers; a pass re-reads the split's K/V).
    for (int m0 = 0; m0 < kv_mul; m0 += kHeadsPerPass) {
        float4 q[kHeadsPerPass];
        float mx[kHeadsPerPass], l[kHeadsPerPass];
        float4 acc[kHeadsPerPass];
        #pragma unroll
        for (int m = 0; m < kHeadsPerPass; ++m) {
            q[m] = (m0 + m < kv_mul && act) ? rope4(a.qkv + (size_t)(kvh * kv_mul + m0 + m) * hs, cs, d0, half)
                                            : make_float4(0, 0, 0, 0);
            mx[m] = -INFINITY;
            l[m] = 0.0f;
            acc[m] = make_float4(0, 0, 0, 0);
        }
        if (mark && m0 == 0) trace_mark(sa, opi, 5);
        for (int tb = t0 + warp * kBatch; tb < t1; tb += GW * kBatch) {
            float4 kk[kBatch], vv[kBatch];
            load_kv_batch<F32>(a, head_base, hs, tb, t1, pos, act, kp, vp, kk, vv);
            #pragma unroll
            for (int m = 0; m < kHeadsPerPass; ++m) {
                if (m0 + m >= kv_mul) break;
                float sc[kBatch];
                float bmax = -INFINITY;
                #pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    // score = q.k / sqrtf(head_size) (src/transformer.c:158-163)
                    const float d = warp_sum(dot4(q[m], kk[j]));
                    sc[j] = (tb + j < t1) ? __fdiv_rn(d, sq) : -INFINITY;
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
        // the group's scratch per (warp, head): max, sum, 2 pad, hs accumulators
        #pragma unroll
        for (int m = 0; m < kHeadsPerPass; ++m) {
            if (m0 + m >= kv_mul) break;
            float *cw = sm + (size_t)(warp * kv_mul + m0 + m) * SW;
            if (lane == 0) {
                cw[0] = mx[m];
                cw[1] = l[m];
            }
            if (act) *reinterpret_cast<float4 *>(cw + 4 + d0) = acc[m];
        }
    }
    const int W = hs + 2;
    if (mark) trace_mark(sa, opi, 6);
    bar_group<GW>(grp);
    for (int m = 0; m < kv_mul; ++m) {
        float M = -INFINITY;
        for (int w = 0; w < GW; ++w) M = fmaxf(M, sm[(size_t)(w * kv_mul + m) * SW]);
        float L = 0.0f;
        for (int w = 0; w < GW; ++w) {
            const float *cw = sm + (size_t)(w * kv_mul + m) * SW;
            L = __fmaf_rn(cw[1], expf(cw[0] - M), L);
        }
        for (int e = gt; e < hs; e += (32 * GW)) {
            float o = 0.0f;
            for (int w = 0; w < GW; ++w) {
                const float *cw = sm + (size_t)(w * kv_mul + m) * SW;
                o = __fmaf_rn(cw[4 + e], expf(cw[0] - M), o);
            }
            if (nsplit == 1) {
                a.out[(size_t)(kvh * kv_mul + m) * hs + e] = __fdiv_rn(o, L);
            } else {
                a.work[((size_t)(kvh * kv_mul + m) * a.max_splits + split) * W + 2 + e] = o;
            }
        }
        if (nsplit > 1 && gt == 0) {
            float *w = a.work + ((size_t)(kvh * kv_mul + m) * a.max_splits + split) * W;
            w[0] = M;
            w[1] = L;
        }
    }
    __threadfence();
    bar_group<GW>(grp);  // the scratch is reused by the next item; every store above is fenced
    if (mark) trace_mark(sa, opi, 7);
    if (nsplit > 1) {
        if (gt == 0) {
            const unsigned ticket = atomicAdd(a.count + kvh, 1u);
            ctl.grp_last[grp] = ticket == (unsigned)nsplit - 1u;
        }
        bar_group<GW>(grp);
        if (!ctl.grp_last[grp]) return;
        __threadfence();
        // Merge the splits: every split's (max, sum) and this thread's accumulators are loaded together
        // (one round trip per kMergeChunk splits), folded with an online rescale.
        for (int m = 0; m < kv_mul; ++m) {
            const float *wb = a.work + (size_t)(kvh * kv_mul + m) * a.max_splits * W;
            float M = -INFINITY, L = 0.0f, o[merge_dims<GW>()];
            #pragma unroll
            for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = 0.0f;
            for (int s0 = 0; s0 < nsplit; s0 += kMergeChunk) {
                float cm[kMergeChunk], cl[kMergeChunk], co[kMergeChunk][merge_dims<GW>()];
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) {
                    const bool in = s0 + j < nsplit;
                    const float *w = wb + (size_t)(s0 + j) * W;
                    cm[j] = in ? __ldcg(w) : -INFINITY;
                    cl[j] = in ? __ldcg(w + 1) : 0.0f;
                    #pragma unroll
                    for (int k = 0; k < merge_dims<GW>(); ++k) {
                        const int e = gt + k * (32 * GW);
                        co[j][k] = (in && e < hs) ? __ldcg(w + 2 + e) : 0.0f;
                    }
                }
                float cmax = M;
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) cmax = fmaxf(cmax, cm[j]);
                const float r = expf(M - cmax);  // 0 while M is -inf
                L = __fmul_rn(L, r);
                #pragma unroll
                for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = __fmul_rn(o[k], r);
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) {
                    const float f = expf(cm[j] - cmax);  // 0 for the padding entries
                    L = __fmaf_rn(cl[j], f, L);
                    #pragma unroll
                    for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = __fmaf_rn(co[j][k], f, o[k]);
                }
                M = cmax;
            }
            #pragma unroll
            for (int k = 0; k < merge_dims<GW>(); ++k) {
                const int e = gt + k * (32 * GW);
                if (e < hs) a.out[(size_t)(kvh * kv_mul + m) * hs + e] = __fdiv_rn(o[k], L);
            }
        }
        if (gt == 0) a.count[kvh] = 0u;
        bar_group<GW>(grp);
    }
    if (gt == 0) red_release_add(done_cnt, (unsigned long long)kv_mul * hs);
}
// The wide form out of line: inlined, its code would share the kernel's register allocation with the
// GEMV consumers and slow every op (measured); a call per CTA-wide item costs little.
template <bool F32>
__device__ __noinline__ void attn_item_wide(const AttnArgs &a, int pos, int kvh, int split, int nsplit, int chunk,
                                            int tid, float *sm, StepCtl &ctl, unsigned long long *done_cnt,
                                            const StepArgs &sa, int opi) {
    attn_item<F32, kAttnWideWarps>(a, pos, kvh, split, nsplit, chunk, 0, tid, sm, ctl, done_cnt, sa, opi);
}

__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const StepArgs sa) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = sa.S, NC = sa.NC;
    uint8_t *ring = smem;
    uint8_t *act = smem + sa.xoff;
    StepCtl &ctl = *reinterpret_cast<StepCtl *>(smem + sa.ctl_off);
    const uint32_t ring_s = smem_u32(ring);

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&ctl.full[i], 1);
            mbar_init(&ctl.empty[i], 1);
        }
        for (int i = 0; i < kStepMaxConsumers * 32; ++i) (&ctl.tok[0][0])[i] = 0xFFFFFFFF00000000ull;  // tag -1
        ctl.abort = 0;
        ctl.last = 0;
        ctl.crit = 1;
        for (int b = 0; b < kStepActBlocks; ++b) ctl.act_ready[b] = 0;
        mbar_fence_init();
    }
    __syncthreads();
    const unsigned long long epoch = *sa.epoch;
    const int pos = *sa.pos;
    const bool pos_ok = pos >= 0 && pos < sa.seq_len;

    if (warp >= kComputeWarps) {
        // ---- producers: stream every GEMV stage of this CTA, op after op ----
        const int q = warp - kComputeWarps;
        if (lane != 0 || !pos_ok) return;
        const uint64_t policy = l2_evict_first_policy();
        int gbase = 0, issued_hi = -1;
        bool ok = true;
        for (int i = 0; i < sa.nops && ok; ++i) {
            const StepOp &op = sa.ops[i];
            if (op.kind == OP_ATTN) {
                // The cache rows this CTA's attention items will read (positions < pos, written by earlier
                // steps) go to L2 now, while the q|k|v GEMV still streams: attention then waits for L2,
                // not behind the weight stream queued at HBM.
                if (q == 0) {
                    const AttnArgs &at = op.at;
                    const int T = pos + 1;
                    int nsplit, chunk;
                    const int groups = kComputeWarps / step_attn_plan(at, T, nsplit, chunk);
                    const size_t row = (size_t)at.head_size * (at.kv_f32 ? 4 : 2);
                    for (int g = 0; g < groups; ++g) {
                        const int it = g * (int)gridDim.x + (int)blockIdx.x;
                        if (it >= at.n_kv_heads * nsplit) break;
                        const int kvh = it / nsplit, t0 = (it % nsplit) * chunk, t1 = min(pos, t0 + chunk);
                        if (t1 <= t0) continue;
                        const size_t off = ((size_t)kvh * at.seq_len + t0) * row;
                        const uint32_t nb = (uint32_t)((size_t)(t1 - t0) * row);
                        bulk_prefetch_l2(static_cast<const uint8_t *>(at.k_cache) + off, nb);
                        bulk_prefetch_l2(static_cast<const uint8_t *>(at.v_cache) + off, nb);
                    }
                }
                continue;
            }
            const Sched sc = op_sched(op);
            // this producer's stages: global index G = gbase + s with G % NP == q
            int s = (q - gbase % kStepProducers + kStepProducers) % kStepProducers;
            for (; s < sc.nst; s += kStepProducers) {
                const int G = gbase + s, slot = G % S;
                if (G >= S && !mbar_wait_abortable(&ctl.empty[slot], (uint32_t)(((G / S) - 1) & 1), op.g.err, &ctl.abort, false)) {
                    ctl.abort = 1;
                    ok = false;
                    break;
                }
                // at most K copies in flight (inflight_crit while the compute warps are in a wait, an
                // activation build or attention; inflight while they consume): stage G - K (this
                // producer's own, issued by it and not yet refilled, so its phase is the slot's latest)
                // must have landed
                const int K = (sa.inflight_crit > 0 && *reinterpret_cast<volatile int *>(&ctl.crit)) ? sa.inflight_crit
                                                                                                : sa.inflight;
                if (K > 0 && G >= K &&
                    !mbar_wait_abortable(&ctl.full[(G - K) % S], (uint32_t)(((G - K) / S) & 1), op.g.err, &ctl.abort, false)) {
                    ctl.abort = 1;
                    ok = false;
                    break;
                }
                {
                    const uint8_t *src = sc.src(op.g.w, s);
                    const size_t packed = (size_t)op.ntiles * op.T * q8_row_bytes(op.g.n);
                    const uint32_t nb = sc.bytes(s);
                    if (!DK_CHK(src >= op.g.w && src + nb <= op.g.w + packed && !((uintptr_t)src & 15) && !(nb & 15) &&
                                    nb <= sa.slot && slot < S,
                                sa.err, 1, G)) {
                        ctl.abort = 1;
                        ok = false;
                        break;
                    }
                }
                mbar_arrive_expect_tx(&ctl.full[slot], sc.bytes(s));
                bulk_g2s(ring + (size_t)slot * sa.slot, sc.src(op.g.w, s), sc.bytes(s), &ctl.full[slot], policy);
                issued_hi = G;
            }
            if (q == 0) trace_mark(sa, i, 3);
            gbase += sc.nst;
        }
        // Never leave a copy in flight into the shared memory of an exiting CTA: wait for the last copy
        // issued into each of this producer's slots.
        for (int G = issued_hi; G >= 0 && G > issued_hi - S; G -= kStepProducers)
            mbar_wait(&ctl.full[G % S], (uint32_t)((G / S) & 1), sa.err);
        return;
    }

    // ---- compute warps ----
    if (!pos_ok) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(sa.err, DK_ERR_INVALID);
        return;
    }
    // op descriptors: op 0 now, op i+1 in registers of threads 32 .. 32+kOpWords-1 during op i
    const bool op_copier = tid >= 32 && tid < 32 + kOpWords;
    if (op_copier) ctl.opbuf[0][tid - 32] = __ldg(reinterpret_cast<const unsigned long long *>(sa.ops) + (tid - 32));
    bar_compute();
    int gbase = 0;
    for (int i = 0; i < sa.nops; ++i) {
        const StepOp &op = *reinterpret_cast<const StepOp *>(ctl.opbuf[i % 3]);
        unsigned long long next_word = 0;
        if (op_copier && i + 1 < sa.nops)
            next_word = __ldg(reinterpret_cast<const unsigned long long *>(sa.ops + i + 1) + (tid - 32));
        if (tid == 0) *reinterpret_cast<volatile int *>(&ctl.crit) = 1;
        if (op.kind == OP_GEMV) {
            const GemvArgs &a = op.g;
            const Sched sc = op_sched(op);
            const bool mine = sc.nst > 0;
            unsigned long long best = 0ull;
            if (a.tagged && a.pro == PRO_RMS_REDUCE && (int)blockIdx.x < a.n_gather) {
                // a gatherer of the tagged exchange, whether or not it owns rows of this op
                const bool gok = tp_gather(a, epoch, tid);
                if (bar_compute_or(!gok || *reinterpret_cast<volatile int *>(&ctl.abort))) break;
            }
            if (mine) {
                float4 nw[4];
                #pragma unroll
                for (int j = 0; j < 4; ++j)
                    nw[j] = (a.norm_w && tid < (a.n >> 4)) ? __ldg(reinterpret_cast<const float4 *>(a.norm_w + 16 * tid) + j)
                                                           : make_float4(0, 0, 0, 0);
                if (op.wait_cnt && tid == 0 && !wait_local(op.wait_cnt, (epoch + 1ull) * op.wait_units, sa.err))
                    ctl.abort = 1;
                if (tid == 0) trace_mark(sa, i, 4);
                // the polling thread's acquire, then this barrier, order every thread's reads
                if (bar_compute_or(*reinterpret_cast<volatile int *>(&ctl.abort))) break;
                if (tid == 0) trace_mark(sa, i, 0);
                int8_t *xq = reinterpret_cast<int8_t *>(act);
                float *xs = reinterpret_cast<float *>(act + ((a.n + 15) & ~15));
                // PRO_F32 (wo, w2): the activation block by block beside the consumers (the same for every
                // thread of the CTA, so every thread takes the same barriers)
                const bool blockwise = a.pro == PRO_F32 && !a.dump_q && ((a.n + 511) >> 9) <= kStepActBlocks;
                const int act_tag = blockwise ? i + 1 : 0;
                if (blockwise) {
                    if (warp >= NC) step_activation_blocks(a, xq, xs, ctl, warp - NC, kComputeWarps - NC, lane, act_tag);
                } else {
                    const int tok = a.pro == PRO_EMB_RMS ? __ldcg(a.tokens + pos) : 0;
                    const bool ok = step_activation(a, tok, xq, xs, ctl, tid, epoch, sc.t0 == 0, nw);
                    if (bar_compute_or(!ok || *reinterpret_cast<volatile int *>(&ctl.abort))) break;
                }
                if (tid == 0) trace_mark(sa, i, 1);
                if (a.dump_q && sc.t0 == 0) {  // diagnostics: the op's input and activation, one CTA
                    const float *src = a.pro == PRO_RMS_REDUCE ? a.x_out : a.x;
                    if (a.tagged && (a.pro == PRO_RMS_REDUCE || a.pro == PRO_EMB_RMS)) {
                        for (int j = tid; j < a.n; j += kComputeThreads)
                            a.dump_in[j] = __uint_as_float((unsigned)__ldcg(a.x64_out + j));
                    } else {
                        for (int j = tid; j < (a.n >> 2); j += kComputeThreads)
                            reinterpret_cast<float4 *>(a.dump_in)[j] = __ldcg(reinterpret_cast<const float4 *>(src) + j);
                    }
                    for (int j = tid; j < (a.n >> 4); j += kComputeThreads)
                        reinterpret_cast<uint4 *>(a.dump_q)[j] = reinterpret_cast<const uint4 *>(xq)[j];
                    for (int j = tid; j < (a.n >> 5); j += kComputeThreads) a.dump_s[j] = xs[j];
                }
                if (tid == 0) *reinterpret_cast<volatile int *>(&ctl.crit) = 0;
                if (warp < NC) {
                    unsigned long long *strace = nullptr;
                    if (sa.stage_trace && i >= sa.stage_op0 && i < sa.stage_op0 + kStageTraceOps &&
                        (int)blockIdx.x < kStageTraceCtas)
                        strace = sa.stage_trace + (((size_t)(i - sa.stage_op0) * kStageTraceCtas + blockIdx.x) *
                                                   kStageTraceStages) * 4;
                    gemv_consume(op, sc, gbase, S, NC, sa.slot, ring_s, smem_u32(xq), smem_u32(xs), ctl, warp, lane, best,
                                 strace, epoch, act_tag);
                    if (a.epi == EPI_ARGMAX) {
                        #pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long other = __shfl_xor_sync(FULL, best, o);
                            best = other > best ? other : best;
                        }
                        if (lane == 0) ctl.wkey[warp] = best;
                    }
                }
                // every row stored, the activation no longer read
                if (bar_compute_or(*reinterpret_cast<volatile int *>(&ctl.abort))) break;
                if (tid == 0) {
                    *reinterpret_cast<volatile int *>(&ctl.crit) = 1;
                    trace_mark(sa, i, 2);
                    const int lo = sc.t0 * op.T, hi = min(a.d, (sc.t0 + sc.nt) * op.T);
                    const unsigned long long rows = hi > lo ? (unsigned long long)(hi - lo) : 0ull;
                    if (a.epi == EPI_PEER && !a.tagged) {
                        // count this CTA's rows on every rank: a rank that sees the count sees the rows
                        __threadfence_system();
                        for (int r = 0; r < a.tp_world; ++r) atomicAdd_system(a.peer_cnt[r], rows);
                    } else if (op.done_cnt) {
                        red_release_add(op.done_cnt, a.epi == EPI_SWIGLU ? rows / 2 : rows);
                    }
                }
            }
            gbase += sc.nst;
            if (a.epi == EPI_ARGMAX) {
                // every CTA takes a ticket; the last one picks the token (src/sampler.c:6-17)
                if (tid == 0) {
                    unsigned long long bb = 0ull;
                    if (mine)
                        for (int w = 0; w < NC; ++w) bb = ctl.wkey[w] > bb ? ctl.wkey[w] : bb;
                    a.amax_part[blockIdx.x] = bb;
                    __threadfence();
                    const unsigned ticket = atomicAdd(a.amax_count, 1u);
                    ctl.last = ticket == gridDim.x - 1;
                }
                bar_compute();
                if (ctl.last && tid == 0) {
                    __threadfence();
                    unsigned long long bb = 0ull;
                    for (int c = 0; c < (int)gridDim.x; ++c) {
                        const unsigned long long kk = __ldcg(a.amax_part + c);
                        bb = kk > bb ? kk : bb;
                    }
                    if (a.tp_world > 1) {
                        for (int r = 0; r < a.tp_world; ++r) a.peer_amax[r][a.tp_rank] = bb;
                        __threadfence_system();
                        for (int r = 0; r < a.tp_world; ++r) atomicAdd_system(a.peer_amax_cnt[r], 1ull);
                        wait_counter(a.amax_keys_cnt, (epoch + 1ull) * (unsigned long long)a.tp_world, a.err);
                        __threadfence();
                        for (int r = 0; r < a.tp_world; ++r) {
                            const unsigned long long k = __ldcg(a.amax_keys + r);
                            bb = k > bb ? k : bb;
                        }
                    }
                    const int vocab = a.vocab > 0 ? a.vocab : a.d;
                    int idx = (bb == 0ull) ? 0 : argmax_idx(bb);
                    if (idx < 0 || idx >= vocab) idx = 0;
                    if (pos + 1 <= a.seq_len && pos + 1 >= *a.n_forced) a.tokens[pos + 1] = idx;
                    *a.amax_count = 0u;
                    __threadfence();
                    *a.pos = pos + 1;
                    *sa.epoch_rw = epoch + 1ull;
                }
            }
        } else {  // OP_ATTN
            const AttnArgs &at = op.at;
            if (op.wait_cnt && tid == 0 && !wait_local(op.wait_cnt, (epoch + 1ull) * op.wait_units, sa.err)) ctl.abort = 1;
            if (tid == 0) trace_mark(sa, i, 4);
            if (bar_compute_or(*reinterpret_cast<volatile int *>(&ctl.abort))) break;
            if (tid == 0) trace_mark(sa, i, 0);
            const int T = pos + 1;
            int nsplit, chunk;
            const int gw = step_attn_plan(at, T, nsplit, chunk);  // the same on every thread
            const int items = at.n_kv_heads * nsplit;
            const int kv_mul = at.n_heads / at.n_kv_heads;
            // item it runs on CTA it % grid: consecutive items (the splits of one head, then the next
            // head) spread over all SMs, so every SM's share of the KV cache is loaded at once
            if (gw == kAttnNarrowWarps) {
                const int grp = warp / kAttnNarrowWarps, gt = tid - grp * 32 * kAttnNarrowWarps;
                float *sm = reinterpret_cast<float *>(act) + (size_t)grp * kAttnNarrowWarps * kv_mul * (at.head_size + 4);
                for (int it = grp * (int)gridDim.x + (int)blockIdx.x; it < items; it += gridDim.x * kAttnGroups) {
                    const int kvh = it / nsplit, split = it % nsplit;
                    if (at.kv_f32)
                        attn_item<true, kAttnNarrowWarps>(at, pos, kvh, split, nsplit, chunk, grp, gt, sm, ctl, op.done_cnt, sa, i);
                    else
                        attn_item<false, kAttnNarrowWarps>(at, pos, kvh, split, nsplit, chunk, grp, gt, sm, ctl, op.done_cnt, sa, i);
                }
            } else {
                float *sm = reinterpret_cast<float *>(act);
                for (int it = (int)blockIdx.x; it < items; it += gridDim.x) {
                    const int kvh = it / nsplit, split = it % nsplit;
                    if (at.kv_f32) attn_item_wide<true>(at, pos, kvh, split, nsplit, chunk, tid, sm, ctl, op.done_cnt, sa, i);
                    else attn_item_wide<false>(at, pos, kvh, split, nsplit, chunk, tid, sm, ctl, op.done_cnt, sa, i);
                }
            }
            bar_compute();  // the scratch (the activation area) is free again
            if (tid == 0) trace_mark(sa, i, 2);
        }
        // the next op's descriptor (its slot last held op i-2, which every thread has left)
        if (op_copier && i + 1 < sa.nops) ctl.opbuf[(i + 1) % 3][tid - 32] = next_word;
        bar_compute();
    }
}

// ---- prompt prefill: the step's own device code over a batch of prompt positions ----------------------
// One CTA per token (the compute warps' layout: 320 threads): the token's Q8_0 activation exactly as the
// decode step builds it (rmsnorm / embedding row / plain quantisation, same reduction order), written
// to xq[t][n], xs[t][n/32] for the tensor-core matmul.  PRO_EMB_RMS also stores the embedding row as
// the token's residual x[t].
__global__ void __launch_bounds__(kComputeThreads) prefill_act_kernel(const GemvArgs a, int ntok, const int *tokens,
                                                                      int8_t *xq_out, float *xs_out) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int t = blockIdx.x, tid = threadIdx.x;
    if (t >= ntok) return;
    const int n = a.n;
    int8_t *xq = reinterpret_cast<int8_t *>(smem);
    float *xs = reinterpret_cast<float *>(smem + ((n + 15) & ~15));
    StepCtl &ctl = *reinterpret_cast<StepCtl *>(smem + gemv_x_bytes_dev(n));
    if (tid == 0) ctl.abort = 0;
    GemvArgs b = a;
    b.x = a.x + (size_t)t * n;  // this token's input row (written back for PRO_EMB_RMS)
    float4 nw[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j)
        nw[j] = (b.norm_w && tid < (n >> 4)) ? __ldg(reinterpret_cast<const float4 *>(b.norm_w + 16 * tid) + j)
                                              : make_float4(0, 0, 0, 0);
    bar_compute();
    const int tok = a.pro == PRO_EMB_RMS ? __ldg(tokens + t) : 0;
    step_activation(b, tok, xq, xs, ctl, tid, 0ull, true, nw);
    bar_compute();
    for (int i = tid; i < n / 16; i += kComputeThreads)
        reinterpret_cast<uint4 *>(xq_out + (size_t)t * n)[i] = reinterpret_cast<const uint4 *>(xq)[i];
    for (int g = tid; g < n / 32; g += kComputeThreads) xs_out[(size_t)t * (n / 32) + g] = xs[g];
}

// RoPE + KV-cache write of every prompt position (grid: tokens x KV heads, one warp): the rotated k and
// the v of position t, rounded to the cache type, exactly as the decode step stores them.
template <bool F32>
__global__ void prefill_kv_kernel(const AttnArgs a, int pos0, int ntok, size_t qkv_stride) {
    const int t = blockIdx.x, kvh = blockIdx.y, lane = threadIdx.x;
    const int hs = a.head_size, half = hs >> 1, d0 = 4 * lane;
    if (t >= ntok || kvh >= a.n_kv_heads || d0 >= hs || pos0 + t >= a.seq_len) return;
    const int dim = a.n_heads * hs, kv_dim = a.n_kv_heads * hs;
    const float *qkv = a.qkv + (size_t)t * qkv_stride;
    const float *cs = a.rope + (size_t)(pos0 + t) * hs;
    const float4 kr = rope4(qkv + dim + (size_t)kvh * hs, cs, d0, half);
    const float4 vr = __ldcg(reinterpret_cast<const float4 *>(qkv + dim + kv_dim + (size_t)kvh * hs + d0));
    const size_t at = (size_t)kvh * a.seq_len * hs + (size_t)(pos0 + t) * hs + d0;
    store_kv4<F32>(a.k_cache, at, kr);
    store_kv4<F32>(a.v_cache, at, vr);
}

// Rows (query head of one position) whose batch scores one warp takes at once: 4 rows x kBatch positions
// = one (row, position) per lane.
constexpr int kPreRowChunk = 4;
static_assert(kPreRowChunk * kBatch == 32, "one score per lane");
constexpr int kPrePartStride = 36;  // floats per (row, position) block of lane partials: 16-byte reads without conflicts

// Attention of the prompt positions of one group (positions that share the decode step's attention form
// and split plan) for one (KV head, split): item = item_base + blockIdx.x, one attention group of GW warps
// (the form's item size: its positions' decode steps run their items on GW warps).  Each K/V
// batch is loaded once and used for every (position, query head) row of the group; each row keeps the
// decode step's own arithmetic (attn_item): the same batches in the same order per warp, the same
// masked tail, the warp merge, the split partials and the last split's merge -- so every output equals
// the decode step's at that position, bit for bit.  The K/V rows of every position up to the group's
// last are in the cache already (prefill_kv_kernel).  State per (warp, row) lives in shared memory:
// [max, sum, -, -, acc[hs]].
// Per K/V batch a warp works on 4 rows at a time in three steps, so that each score's scalar work is
// done once instead of on all 32 lanes:
//   (a) lanes over head dims: each lane's 4-dim partial dot of every (row, position) -> shared memory;
//   (b) one lane per (row, position): the 32 partials summed in warp_sum's butterfly order (at step o,
//       v[l] = v[l] + v[l + o]: the value every lane of warp_sum ends with), the division by sqrt(hs),
//       the batch max over the row's 8 lanes, the rescale and exp, and the running sum in position order
//       through shuffles;
//   (c) lanes over head dims: acc = acc * rescale, then acc = fma(p_j, v_j, acc) in position order.
template <bool F32, int GW>
__global__ void __launch_bounds__(32 * GW, GW == kAttnNarrowWarps ? 8 : 2)
    prefill_attn_kernel(const AttnArgs a, int pos0, const PrefillGroup *groups, int ngroups, long long item_base,
                        size_t qkv_stride, size_t out_stride, size_t work_stride, size_t count_stride) {
    extern __shared__ __align__(16) float psm[];
    __shared__ int last_split[kPrefillRows];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hs = a.head_size, half = hs >> 1, d0 = 4 * lane;
    const bool act = d0 < hs;
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const long long item = item_base + blockIdx.x;
    int lo = 0, hi = ngroups - 1;  // the group holding this item: the last with item0 <= item
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (groups[mid].item0 <= item) lo = mid;
        else hi = mid - 1;
    }
    const PrefillGroup g = groups[lo];
    const int it = (int)(item - g.item0), kvh = it / g.nsplit, split = it % g.nsplit;
    const int rows = g.count * kv_mul;
    if (kvh >= a.n_kv_heads || rows > kPrefillRows || g.first < pos0) return;
    const int t0 = split * g.chunk, tmax = min(g.first + g.count, t0 + g.chunk);
    const int SW = hs + 4, W = hs + 2;
    float *qs = psm;                           // [kPrefillRows][hs]
    float *stt = psm + (size_t)kPrefillRows * hs;  // [GW][kPrefillRows][SW]
    for (int r = warp; r < rows; r += GW) {
        const int q = r / kv_mul, m = r % kv_mul, pos = g.first + q;
        if (act)
            *reinterpret_cast<float4 *>(qs + (size_t)r * hs + d0) =
                rope4(a.qkv + (size_t)(pos - pos0) * qkv_stride + (size_t)(kvh * kv_mul + m) * hs,
                      a.rope + (size_t)pos * hs, d0, half);
    }
    for (int r = 0; r < rows; ++r) {
        float *sw = stt + ((size_t)warp * kPrefillRows + r) * SW;
        if (lane == 0) {
            sw[0] = -INFINITY;
            sw[1] = 0.0f;
        }
        if (act) *reinterpret_cast<float4 *>(sw + 4 + d0) = make_float4(0, 0, 0, 0);
    }
    __syncthreads();
    const float sq = __fsqrt_rn((float)hs);
    const size_t head_base = (size_t)kvh * a.seq_len * hs + d0;
    float *part = psm + (size_t)kPrefillRows * hs + (size_t)GW * kPrefillRows * SW +
                  (size_t)warp * kPreRowChunk * kBatch * kPrePartStride;  // this warp's [32][36] partials
    float *pjs = psm + (size_t)kPrefillRows * hs + (size_t)GW * kPrefillRows * SW +
                 (size_t)GW * kPreRowChunk * kBatch * kPrePartStride + (size_t)warp * 40;  // [4][8], [4]
    auto row_end = [&](int r) { return min(g.first + r / kv_mul + 1, t0 + g.chunk); };
    for (int tb = t0 + warp * kBatch; tb < tmax; tb += GW * kBatch) {
        float4 kk[kBatch], vv[kBatch];
        #pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int t = tb + j;
            kk[j] = (t < tmax && act) ? load_kv4<F32>(a.k_cache, head_base + (size_t)t * hs) : make_float4(0, 0, 0, 0);
            vv[j] = (t < tmax && act) ? load_kv4<F32>(a.v_cache, head_base + (size_t)t * hs) : make_float4(0, 0, 0, 0);
        }
        for (int rc = 0; rc < rows; rc += kPreRowChunk) {
            const int nr = min(kPreRowChunk, rows - rc);
            // (a) partial dots: part[rr * 8 + j][lane]
            for (int rr = 0; rr < nr; ++rr) {
                if (tb >= row_end(rc + rr)) continue;  // the decode step's warp has left its loop for this row
                const float4 qv =
                    act ? *reinterpret_cast<const float4 *>(qs + (size_t)(rc + rr) * hs + d0) : make_float4(0, 0, 0, 0);
                #pragma unroll
                for (int j = 0; j < kBatch; ++j) part[(rr * kBatch + j) * kPrePartStride + lane] = dot4(qv, kk[j]);
            }
            __syncwarp();
            // (b) lane = rr * 8 + j
            {
                const int rr = lane >> 3, j = lane & 7, r = rc + rr;
                const int t1 = rr < nr ? row_end(r) : 0;
                const bool live = rr < nr && tb < t1;  // the same on the row's 8 lanes
                float v[32];
                const float4 *pv = reinterpret_cast<const float4 *>(part + lane * kPrePartStride);
                #pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 f = pv[i];
                    v[4 * i] = f.x;
                    v[4 * i + 1] = f.y;
                    v[4 * i + 2] = f.z;
                    v[4 * i + 3] = f.w;
                }
                #pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    #pragma unroll
                    for (int l = 0; l < o; ++l) v[l] = __fadd_rn(v[l], v[l + o]);
                }
                // score = q.k / sqrtf(head_size) (src/transformer.c:158-163)
                const float sc = (live && tb + j < t1) ? __fdiv_rn(v[0], sq) : -INFINITY;
                float bmax = sc;
                bmax = fmaxf(bmax, __shfl_xor_sync(FULL, bmax, 4));
                bmax = fmaxf(bmax, __shfl_xor_sync(FULL, bmax, 2));
                bmax = fmaxf(bmax, __shfl_xor_sync(FULL, bmax, 1));
                float *sw = stt + ((size_t)warp * kPrefillRows + (live ? r : 0)) * SW;
                const float mx = live ? sw[0] : 0.0f, l = live ? sw[1] : 0.0f;
                const float mnew = fmaxf(mx, bmax);
                const float rescale = expf(mx - mnew);
                const float pj = expf(sc - mnew);
                float lm = __fmul_rn(l, rescale);
                #pragma unroll
                for (int jj = 0; jj < kBatch; ++jj) lm = __fadd_rn(lm, __shfl_sync(FULL, pj, (lane & ~7) + jj));
                __syncwarp();
                if (live) {
                    pjs[rr * kBatch + j] = pj;
                    if (j == 0) {
                        pjs[kPreRowChunk * kBatch + rr] = rescale;
                        sw[0] = mnew;
                        sw[1] = lm;
                    }
                }
            }
            __syncwarp();
            // (c) acc = acc * rescale, then fma(p_j, v_j, acc); positions at or past t1 are zero rows
            for (int rr = 0; rr < nr; ++rr) {
                const int r = rc + rr, t1 = row_end(r);
                if (tb >= t1) continue;
                float *sw = stt + ((size_t)warp * kPrefillRows + r) * SW;
                if (act) {
                    const float rescale = pjs[kPreRowChunk * kBatch + rr];
                    float4 am = *reinterpret_cast<const float4 *>(sw + 4 + d0);
                    am = make_float4(__fmul_rn(am.x, rescale), __fmul_rn(am.y, rescale), __fmul_rn(am.z, rescale),
                                     __fmul_rn(am.w, rescale));
                    #pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        const float pj = pjs[rr * kBatch + j];
                        const float4 vj = (tb + j < t1) ? vv[j] : make_float4(0, 0, 0, 0);
                        am.x = __fmaf_rn(pj, vj.x, am.x);
                        am.y = __fmaf_rn(pj, vj.y, am.y);
                        am.z = __fmaf_rn(pj, vj.z, am.z);
                        am.w = __fmaf_rn(pj, vj.w, am.w);
                    }
                    *reinterpret_cast<float4 *>(sw + 4 + d0) = am;
                }
            }
            __syncwarp();
        }
    }
    __syncthreads();
    // the warps' merge, per row (attn_item's order), then the output or this split's partial
    for (int r = 0; r < rows; ++r) {
        const int q = r / kv_mul, m = r % kv_mul, pos = g.first + q;
        const float *s0 = stt + (size_t)r * SW;
        float M = -INFINITY;
        for (int w = 0; w < GW; ++w) M = fmaxf(M, s0[(size_t)w * kPrefillRows * SW]);
        float L = 0.0f;
        for (int w = 0; w < GW; ++w) {
            const float *cw = s0 + (size_t)w * kPrefillRows * SW;
            L = __fmaf_rn(cw[1], expf(cw[0] - M), L);
        }
        const size_t hrow = (size_t)(kvh * kv_mul + m);
        for (int e = tid; e < hs; e += (32 * GW)) {
            float o = 0.0f;
            for (int w = 0; w < GW; ++w) {
                const float *cw = s0 + (size_t)w * kPrefillRows * SW;
                o = __fmaf_rn(cw[4 + e], expf(cw[0] - M), o);
            }
            if (g.nsplit == 1) a.out[(size_t)(pos - pos0) * out_stride + hrow * hs + e] = __fdiv_rn(o, L);
            else a.work[(size_t)(pos - pos0) * work_stride + (hrow * a.max_splits + split) * W + 2 + e] = o;
        }
        if (g.nsplit > 1 && tid == 0) {
            float *w = a.work + (size_t)(pos - pos0) * work_stride + (hrow * a.max_splits + split) * W;
            w[0] = M;
            w[1] = L;
        }
    }
    if (g.nsplit == 1) return;
    __threadfence();
    __syncthreads();
    if (tid < g.count) {
        const unsigned ticket = atomicAdd(a.count + (size_t)(g.first + tid - pos0) * count_stride + kvh, 1u);
        last_split[tid] = ticket == (unsigned)g.nsplit - 1u;
    }
    __syncthreads();
    // the last split of a position merges its splits (attn_item's merge)
    for (int q = 0; q < g.count; ++q) {
        if (!last_split[q]) continue;
        __threadfence();
        const int pos = g.first + q;
        const float *work = a.work + (size_t)(pos - pos0) * work_stride;
        for (int m = 0; m < kv_mul; ++m) {
            const float *wb = work + (size_t)(kvh * kv_mul + m) * a.max_splits * W;
            float M = -INFINITY, L = 0.0f, o[merge_dims<GW>()];
            #pragma unroll
            for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = 0.0f;
            for (int s0 = 0; s0 < g.nsplit; s0 += kMergeChunk) {
                float cm[kMergeChunk], cl[kMergeChunk], co[kMergeChunk][merge_dims<GW>()];
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) {
                    const bool in = s0 + j < g.nsplit;
                    const float *w = wb + (size_t)(s0 + j) * W;
                    cm[j] = in ? __ldcg(w) : -INFINITY;
                    cl[j] = in ? __ldcg(w + 1) : 0.0f;
                    #pragma unroll
                    for (int k = 0; k < merge_dims<GW>(); ++k) {
                        const int e = tid + k * (32 * GW);
                        co[j][k] = (in && e < hs) ? __ldcg(w + 2 + e) : 0.0f;
                    }
                }
                float cmax = M;
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) cmax = fmaxf(cmax, cm[j]);
                const float rr = expf(M - cmax);
                L = __fmul_rn(L, rr);
                #pragma unroll
                for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = __fmul_rn(o[k], rr);
                #pragma unroll
                for (int j = 0; j < kMergeChunk; ++j) {
                    const float f = expf(cm[j] - cmax);
                    L = __fmaf_rn(cl[j], f, L);
                    #pragma unroll
                    for (int k = 0; k < merge_dims<GW>(); ++k) o[k] = __fmaf_rn(co[j][k], f, o[k]);
                }
                M = cmax;
            }
            #pragma unroll
            for (int k = 0; k < merge_dims<GW>(); ++k) {
                const int e = tid + k * (32 * GW);
                if (e < hs) a.out[(size_t)(pos - pos0) * out_stride + (size_t)(kvh * kv_mul + m) * hs + e] = __fdiv_rn(o[k], L);
            }
        }
        if (tid == 0) a.count[(size_t)(pos - pos0) * count_stride + kvh] = 0u;
    }
}

}  // namespace

namespace {

// ---- tensor-parallel prefill exchange ----------------------------------------------------------------
// The partial rows of wo / w2 (this rank's columns), stored to every rank's receive area with plain
// peer stores, then a system-scope fence so that a rank that sees the counter sees the rows.
__global__ void prefill_scatter_kernel(const float4 *src, float *const *dst, int world, size_t off, size_t n4) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldcg(src + i);
        for (int q = 0; q < world; ++q) reinterpret_cast<float4 *>(dst[q] + off)[i] = v;
    }
    __threadfence_system();
}
__global__ void prefill_signal_kernel(unsigned long long *const *cnt, int world) {
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < world; ++q) atomicAdd_system(cnt[q], 1ull);
    }
}
__global__ void prefill_wait_kernel(const unsigned long long *cnt, unsigned long long target, int *err) {
    if (threadIdx.x == 0 && !wait_counter(cnt, target, err)) atomicOr(err, DK_ERR_COMM);
}
// x + (partial_0 + partial_1 + ...), ranks in order: the decode step's reduce prologue, element by element.
__global__ void prefill_reduce_kernel(float4 *x, const float4 *recv, size_t stride4, int world, size_t n4) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 t = __ldcg(recv + i);
        for (int q = 1; q < world; ++q) {
            const float4 u = __ldcg(recv + (size_t)q * stride4 + i);
            t = make_float4(__fadd_rn(t.x, u.x), __fadd_rn(t.y, u.y), __fadd_rn(t.z, u.z), __fadd_rn(t.w, u.w));
        }
        const float4 v = x[i];
        x[i] = make_float4(__fadd_rn(v.x, t.x), __fadd_rn(v.y, t.y), __fadd_rn(v.z, t.z), __fadd_rn(v.w, t.w));
    }
}

}  // namespace

cudaError_t launch_prefill_scatter(const float *src, float *const *dst, int world, size_t off, size_t nf, cudaStream_t st) {
    if (nf % 4 || off % 4 || world < 1 || world > 8) return cudaErrorInvalidValue;
    const size_t n4 = nf / 4;
    const unsigned blocks = (unsigned)std::min<size_t>((n4 + 255) / 256, 4096);
    prefill_scatter_kernel<<<blocks ? blocks : 1, 256, 0, st>>>(reinterpret_cast<const float4 *>(src), dst, world, off, n4);
    return cudaGetLastError();
}
cudaError_t launch_prefill_signal(unsigned long long *const *cnt, int world, cudaStream_t st) {
    prefill_signal_kernel<<<1, 32, 0, st>>>(cnt, world);
    return cudaGetLastError();
}
cudaError_t launch_prefill_wait(const unsigned long long *cnt, unsigned long long target, int *err, cudaStream_t st) {
    prefill_wait_kernel<<<1, 32, 0, st>>>(cnt, target, err);
    return cudaGetLastError();
}
cudaError_t launch_prefill_reduce(float *x, const float *recv, size_t stride, int world, size_t nf, cudaStream_t st) {
    if (nf % 4 || stride % 4) return cudaErrorInvalidValue;
    const size_t n4 = nf / 4;
    const unsigned blocks = (unsigned)std::min<size_t>((n4 + 255) / 256, 4096);
    prefill_reduce_kernel<<<blocks ? blocks : 1, 256, 0, st>>>(reinterpret_cast<float4 *>(x),
                                                               reinterpret_cast<const float4 *>(recv), stride / 4, world, n4);
    return cudaGetLastError();
}

int prefill_attn_plan(const AttnArgs &a, int pos0, int ntok, PrefillGroup *groups, long long *items,
                      long long *narrow_items) {
    const int kv_mul = a.n_heads / a.n_kv_heads;
    const int qmax = std::max(1, kPrefillRows / kv_mul);
    int n = 0;
    long long total = 0, narrow = 0;
    for (int t = 0; t < ntok; ++t) {
        const int pos = pos0 + t, T = pos + 1;
        int ns, ch;
        const int gw = step_attn_plan(a, T, ns, ch);
        if (n > 0) {
            PrefillGroup &b = groups[n - 1];
            // the same form; one split: the run is [0, T) whatever the chunk; more: the same chunk, the same
            // split starts
            if (b.count < qmax && b.warps == gw && b.nsplit == ns && (ns == 1 || b.chunk == ch)) {
                ++b.count;
                if (ns == 1) b.chunk = T;
                continue;
            }
            total += (long long)a.n_kv_heads * b.nsplit;
        }
        groups[n].first = pos;
        groups[n].count = 1;
        groups[n].nsplit = ns;
        groups[n].chunk = ch;
        groups[n].item0 = (int)total;
        groups[n].warps = gw;
        if (gw == kAttnNarrowWarps) narrow = total + (long long)a.n_kv_heads * ns;
        ++n;
    }
    if (n > 0) total += (long long)a.n_kv_heads * groups[n - 1].nsplit;
    if (items) *items = total;
    if (narrow_items) *narrow_items = narrow;
    return n;
}

cudaError_t launch_prefill_act(const GemvArgs &a, int ntok, const int *tokens, int8_t *xq, float *xs, cudaStream_t st) {
    const size_t smem = gemv_x_bytes(a.n) + ((sizeof(StepCtl) + 127) & ~(size_t)127);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(prefill_act_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    prefill_act_kernel<<<ntok, kComputeThreads, smem, st>>>(a, ntok, tokens, xq, xs);
    return cudaGetLastError();
}

cudaError_t launch_prefill_kv(const AttnArgs &a, int pos0, int ntok, size_t qkv_stride, cudaStream_t st) {
    dim3 grid(ntok, a.n_kv_heads);
    if (a.kv_f32) prefill_kv_kernel<true><<<grid, 32, 0, st>>>(a, pos0, ntok, qkv_stride);
    else prefill_kv_kernel<false><<<grid, 32, 0, st>>>(a, pos0, ntok, qkv_stride);
    return cudaGetLastError();
}

template <bool F32, int GW>
static cudaError_t launch_prefill_attn_form(const AttnArgs &a, int pos0, const PrefillGroup *d_groups, int ngroups,
                                            long long item0, long long items, size_t qkv_stride, size_t out_stride,
                                            size_t work_stride, size_t count_stride, cudaStream_t st) {
    if (items <= 0) return cudaSuccess;
    const size_t smem = sizeof(float) * ((size_t)kPrefillRows * a.head_size +
                                         (size_t)GW * kPrefillRows * (a.head_size + 4) +
                                         (size_t)GW * kPreRowChunk * kBatch * kPrePartStride + (size_t)GW * 40);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<F32, GW>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    prefill_attn_kernel<F32, GW><<<(unsigned)items, 32 * GW, smem, st>>>(a, pos0, d_groups, ngroups, item0, qkv_stride,
                                                                        out_stride, work_stride, count_stride);
    return cudaGetLastError();
}

cudaError_t launch_prefill_attn(const AttnArgs &a, int pos0, const PrefillGroup *d_groups, int ngroups,
                                long long items, long long narrow_items, size_t qkv_stride, size_t out_stride,
                                size_t work_stride, size_t count_stride, cudaStream_t st) {
    if (ngroups < 1 || items < 1 || items > 0x7FFFFFFFLL || narrow_items < 0 || narrow_items > items ||
        a.head_size > 128 || a.head_size % 4)
        return cudaErrorInvalidValue;
    // the narrow groups' items first (the positions before wide_from), then the wide ones'
    cudaError_t e;
    if (a.kv_f32) {
        e = launch_prefill_attn_form<true, kAttnNarrowWarps>(a, pos0, d_groups, ngroups, 0, narrow_items, qkv_stride,
                                                             out_stride, work_stride, count_stride, st);
        if (e == cudaSuccess)
            e = launch_prefill_attn_form<true, kAttnWideWarps>(a, pos0, d_groups, ngroups, narrow_items,
                                                               items - narrow_items, qkv_stride, out_stride,
                                                               work_stride, count_stride, st);
    } else {
        e = launch_prefill_attn_form<false, kAttnNarrowWarps>(a, pos0, d_groups, ngroups, 0, narrow_items, qkv_stride,
                                                              out_stride, work_stride, count_stride, st);
        if (e == cudaSuccess)
            e = launch_prefill_attn_form<false, kAttnWideWarps>(a, pos0, d_groups, ngroups, narrow_items,
                                                                items - narrow_items, qkv_stride, out_stride,
                                                                work_stride, count_stride, st);
    }
    return e;
}

size_t step_ctl_bytes() { return (sizeof(StepCtl) + 127) & ~(size_t)127; }
size_t step_attn_scratch_bytes(int n_heads, int n_kv_heads, int head_size) {
    return sizeof(float) * (size_t)kComputeWarps * (n_heads / n_kv_heads) * (head_size + 4);
}
int step_attn_item_slots(int num_ctas, int warps) { return num_ctas * (kComputeWarps / warps); }
int step_threads() { return kStepThreads; }

cudaError_t launch_step(const StepArgs &sa, int grid, cudaStream_t st) {
    if (sa.S < 1 || sa.S > kStepMaxSlots || sa.S < kStepProducers || sa.S % kStepProducers || sa.NC < 1 ||
        sa.NC > kStepMaxConsumers || sa.NC > kComputeWarps || sa.S < 2 * sa.NC + 2 || sa.inflight < 0 || sa.inflight % kStepProducers || sa.inflight > sa.S ||
        sa.inflight_crit < 0 || sa.inflight_crit % kStepProducers || sa.inflight_crit > sa.S || sa.smem > 227 * 1024 ||
        sa.ctl_off + step_ctl_bytes() > sa.smem || sa.xoff < (size_t)sa.S * sa.slot || sa.ctl_off < sa.xoff)
        return cudaErrorInvalidValue;
    static int attr_bytes[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (attr_bytes[dev] < (int)sa.smem) {
        cudaError_t e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sa.smem);
        if (e != cudaSuccess) return e;
        attr_bytes[dev] = (int)sa.smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = sa.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the counter waits need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, step_kernel, sa);
}

int step_max_ctas_per_sm(size_t smem) {
    int n = 0;
    if (cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, step_kernel, kStepThreads, smem) != cudaSuccess) return 0;
    return n;
}

}  // namespace dk
