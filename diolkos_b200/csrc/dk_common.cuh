// dk_common.cuh -- device helpers shared by the Diolkos B200 kernels (sm_100a only).
//
// Inline PTX wrappers for the Blackwell features the kernels use: mbarriers, the bulk-copy
// engine (cp.async.bulk, TMA without a tensor map), programmatic dependent launch
// (griddepcontrol) and L2 cache-policy hints.  Every wait on an mbarrier or a flag is bounded:
// after DK_WAIT_LIMIT_CYCLES the waiter records DK_ERR_TIMEOUT in the error word that every
// kernel receives and gives up, so a logic error can never hang the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/diolkos.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "diolkos_b200 kernels are written for sm_100a only"
#endif

namespace dk {

constexpr unsigned FULL = 0xffffffffu;
// ~0.5 s at 2 GHz: every legitimate wait in these kernels completes within microseconds.
constexpr long long DK_WAIT_LIMIT_CYCLES = 1000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
// Make the initialised barriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns false (after recording
// DK_ERR_TIMEOUT) if the limit is reached.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
            atomicOr(err, DK_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait that also gives up as soon as another warp of the CTA has raised *abort.  spin = poll
// with test_wait (lowest wake-up latency, for short hand-offs) instead of the suspending try_wait.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t *bar, uint32_t parity, int *err, const int *abort,
                                                    bool spin) {
    if (spin ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (spin ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<const volatile int *>(abort)) return false;
        if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
            atomicOr(err, DK_ERR_TIMEOUT);
            return false;
        }
    }
}

// ---- cross-GPU signalling (tensor parallel, over NVLink peer memory) -----------------------------
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until the counter (written by other GPUs) reaches `target`.  A peer that never
// arrives raises DK_ERR_COMM after DK_WAIT_LIMIT_CYCLES instead of hanging the kernel.
__device__ __forceinline__ bool wait_counter(const unsigned long long *cnt, unsigned long long target, int *err) {
    if (ld_acquire_sys(cnt) >= target) return true;
    const long long t0 = clock64();
    while (ld_acquire_sys(cnt) < target) {
        if (clock64() - t0 > DK_WAIT_LIMIT_CYCLES) {
            atomicOr(err, DK_ERR_COMM);
            return false;
        }
    }
    return true;
}

// ---- bulk copy engine (TMA, 1-D) --------------------------------------------------------------
// L2 policy for streamed-once data (weights): evict first, so the KV cache and activations stay.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Global -> shared bulk copy completing on `bar`.  dst, src 16-byte aligned; bytes % 16 == 0.
// No cluster multicast: the source is always this GPU's own memory and the copy lands in this
// CTA's shared memory only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before its later async-proxy
// (bulk-copy) accesses: used before a copy overwrites a slot that threads just read.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Ask the bulk-copy engine to bring [src, src+bytes) into L2 (no shared memory, no completion
// signal).  src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- programmatic dependent launch ------------------------------------------------------------
// Wait until the preceding kernel in the stream has completed and its writes are visible.  Every
// kernel calls this before it reads anything an earlier kernel wrote or writes anything an
// earlier kernel reads; only reads of constant data (weights, tables) may precede it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to be scheduled (its pre-wait prologue may then overlap
// with the rest of this kernel).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- shared-memory loads through 32-bit shared addresses ---------------------------------------
// Explicit ld.shared: a load through a generic pointer that the compiler cannot prove to be shared
// is issued as a generic load and waited on like a global one.
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

// ---- small helpers ------------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// The Q8_0 quantisation of one value given the group's reciprocal scale: rint(x * inv), round
// half to even (the reference's nearbyintf in the default rounding mode).  A non-finite product
// (an all-zero group gives 0*inf = NaN; a denormal scale overflows inv to inf) converts to 0, which
// is what the reference's int8 cast yields on x86 (the conversion returns INT_MIN, low byte 0).
__device__ __forceinline__ int q8_round(float x, float inv) {
    const float v = __fmul_rn(x, inv);
    return fabsf(v) <= 128.0f ? __float2int_rn(v) : 0;
}
// Group scale and its reciprocal from the group's max |x|: scale = amax * (1/127) rounded,
// inv = 1/scale exactly rounded -- what the reference's -Ofast build computes
// (src/tensor.c:213-226 and :327-339).
__device__ __forceinline__ void q8_scale(float amax, float &scale, float &inv) {
    scale = __fmul_rn(amax, 1.0f / 127.0f);
    inv = __frcp_rn(scale);
}

__device__ __forceinline__ int dp4a_16B(const uint4 &a, const uint4 &b) {
    int acc = __dp4a(static_cast<int>(a.x), static_cast<int>(b.x), 0);
    acc = __dp4a(static_cast<int>(a.y), static_cast<int>(b.y), acc);
    acc = __dp4a(static_cast<int>(a.z), static_cast<int>(b.z), acc);
    acc = __dp4a(static_cast<int>(a.w), static_cast<int>(b.w), acc);
    return acc;
}

}  // namespace dk
