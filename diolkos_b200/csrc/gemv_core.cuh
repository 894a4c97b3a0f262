// gemv_core.cuh -- the per-stage arithmetic of the Q8_0 GEMV (reference matmul_Q8_0,
// src/utils.c:106-138), shared by the standalone GEMV kernel (gemv.cu) and the persistent decode-step
// kernel (step.cu): loading a row's segment and the activation from shared memory, the exact group
// terms (float)dot * (w_scale * x_scale), the warp-to-warp hand-off of running row sums, and the
// greedy-token keys.
#pragma once

#include "dk_common.cuh"
#include "dk_kernels.h"

namespace dk {

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    if (v != v) u = 0u;  // NaN never wins (the reference's strict '>' never selects it)
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}
__device__ __forceinline__ int argmax_idx(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
}

// Data of 4 consecutive groups of one row: the 4 weight scales, the 4 activation scales, the 8
// 16-byte weight chunks and the 8 16-byte activation chunks.
struct Quad {
    uint4 s;
    float4 xs;
    uint4 w[8], x[8];
};

// Load quad q (groups 4q..4q+3) of a full 512-column segment.  seg, xq, xs are 32-bit shared-memory
// addresses of the row's segment and of this block's activation values/scales.
__device__ __forceinline__ void load_quad(Quad &d, int q, uint32_t seg, uint32_t xq, uint32_t xs, int r) {
    d.s = lds128(seg + 512 + 16 * q8_swz_s(q, r, 512));
    d.xs = lds_f4(xs + 16 * q);
    #pragma unroll
    for (int c = 0; c < 8; ++c) {
        d.w[c] = lds128(seg + 16 * q8_swz_q(8 * q + c, r, 512));
        d.x[c] = lds128(xq + 128 * q + 16 * c);
    }
}

// Wait until this lane's token word carries stage G's tag, then take the running sum from it.  Every
// lane polls its own word: one shared-memory round trip when the sums have landed, which is what the
// hand-off costs on the row sums' serial path (the warp's 32 words are two wavefronts).  A word is
// single-copy atomic, so the sum and its tag arrive together: no fence, no separate flag.  The abort
// flag and the clock are looked at every 16 polls only, so a poll is one load.  Bounded.
__device__ __forceinline__ bool lane_token_wait(const unsigned long long *row0, int lane, int G, float &sum, int *err,
                                                const int *abort) {
    const volatile unsigned long long *p = row0 + lane;
    unsigned long long v = *p;
    if ((unsigned)(v >> 32) == (unsigned)G) {
        sum = __uint_as_float((unsigned)v);
        return true;
    }
    const long long t0 = clock64();
    for (int k = 1;; ++k) {
        v = *p;
        if ((unsigned)(v >> 32) == (unsigned)G) {
            sum = __uint_as_float((unsigned)v);
            return true;
        }
        if (!(k & 15)) {
            if (*reinterpret_cast<const volatile int *>(abort)) return false;
            if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
                atomicOr(err, DK_ERR_TIMEOUT);
                return false;
            }
        }
    }
}

// The 16 terms (float)dot_g * (ws_g * xs_g) of one row over one full block, each rounded exactly as
// in the reference's loop.  Loads of quad q+1 are issued before quad q's arithmetic.
__device__ __forceinline__ void quad_terms(float *t, const Quad &d) {
    const float ws[4] = {__uint_as_float(d.s.x), __uint_as_float(d.s.y), __uint_as_float(d.s.z), __uint_as_float(d.s.w)};
    const float xs[4] = {d.xs.x, d.xs.y, d.xs.z, d.xs.w};
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int dot = dp4a_16B(d.w[2 * j + 1], d.x[2 * j + 1]) + dp4a_16B(d.w[2 * j], d.x[2 * j]);
        t[j] = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws[j], xs[j]));
    }
}
__device__ __forceinline__ void block_terms_full(float *t, uint32_t seg, uint32_t xq, uint32_t xs, int r) {
    Quad A;
    load_quad(A, 0, seg, xq, xs, r);
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
        Quad B;
        if (q < 3) load_quad(B, q + 1, seg, xq, xs, r);
        quad_terms(t + 4 * q, A);
        if (q < 3) A = B;
    }
}
// Partial last block: wb/32 < 16 groups.
__device__ __forceinline__ void block_terms_part(float *t, uint32_t seg, uint32_t xq, uint32_t xs, int wb, int r) {
    const int ng = wb >> 5;
    const uint32_t scp = seg + wb;
    #pragma unroll
    for (int g = 0; g < 16; ++g) {
        if (g >= ng) break;
        const float ws = lds_f32(scp + 16 * q8_swz_s(g >> 2, r, wb) + 4 * (g & 3));
        const float xsg = lds_f32(xs + 4 * g);
        const uint4 w0 = lds128(seg + 16 * q8_swz_q(2 * g, r, wb));
        const uint4 w1 = lds128(seg + 16 * q8_swz_q(2 * g + 1, r, wb));
        const uint4 x0 = lds128(xq + 32 * g), x1 = lds128(xq + 32 * g + 16);
        const int dot = dp4a_16B(w1, x1) + dp4a_16B(w0, x0);
        t[g] = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, xsg));
    }
}

struct Sched {  // the CTA's stages: tile t0 + s / nblk, block s % nblk, for s < nst
    int t0, nt, nblk, T, n, nst;
    size_t tile_bytes;
    __device__ const uint8_t *src(const uint8_t *base, int s) const {
        return base + (size_t)(t0 + s / nblk) * tile_bytes + (size_t)T * 576 * (s % nblk);
    }
    __device__ uint32_t bytes(int s) const { return (uint32_t)((size_t)T * q8_blk_bytes(q8_blk_width(n, s % nblk))); }
};

}  // namespace dk
