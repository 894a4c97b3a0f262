// gemm.cu -- the Q8_0 matmul for a BATCH of activation vectors (prompt prefill: the reference runs
// matmul_Q8_0, src/utils.c:106-138, once per prompt token) on the 5th-generation tensor cores.
//
//   out[t][i] = sum over groups g, in order, of (float)dot_g(W[i], x_t) * (w_scale[i][g] * x_scale[t][g])
//
// which is the GEMV's arithmetic exactly: every output equals what the GEMV gives for token t, bit for
// bit.  The int32 group dots are the GEMM part; they come from tcgen05.mma.kind::i8 with K = 32, ONE
// MMA PER GROUP into its own TMEM accumulator (s32, no accumulation across groups), so the fp32 sum
// over groups stays in the reference's order in the epilogue.
//
// CTA = 128 weight rows (M) x 32 tokens (N); 128 threads, thread m owns row m.  Per 512-column block:
//  * all threads copy the block's weight values (from the packed tile layout, de-swizzled) and the
//    tokens' activation values into shared memory in the canonical K-major no-swizzle layout
//    (8-row x 16-byte core matrices), and the scales beside them;
//  * one thread issues the block's (up to) 16 MMAs -- group g's 128x32 int8 tile against the tokens'
//    32x32 tile, into TMEM columns [32g, 32g+32) -- and commits them to an mbarrier;
//  * every thread waits, reads its row's dots for each group (tcgen05.ld 32x32b: lane = row, column =
//    token) and folds term = (float)dot * (ws * xs) into its 32 running sums in group order.
// The epilogue then stores / adds (residual) / applies SwiGLU to the 32 sums.
//
// Every wait is bounded; a CTA that gives up still frees its TMEM.
#include "dk_common.cuh"
#include "dk_kernels.h"

namespace dk {
namespace {

constexpr int kGemmM = 128;      // weight rows per CTA (one per thread; the MMA's M)
constexpr int kGemmN = 32;       // tokens per CTA (the MMA's N)
constexpr int kGemmThreads = 128;
constexpr int kGroupsPerBlock = 16;
constexpr uint32_t kTmemCols = kGroupsPerBlock * kGemmN;  // 512: one 32-column accumulator per group
// shared memory: A[16 groups][128 x 32 B], B[16][32 x 32 B], ws[16][128], xs[16][32], mbarrier, TMEM slot
constexpr size_t kAOff = 0, kABytes = (size_t)kGroupsPerBlock * kGemmM * 32;
constexpr size_t kBOff = kAOff + kABytes, kBBytes = (size_t)kGroupsPerBlock * kGemmN * 32;
constexpr size_t kWsOff = kBOff + kBBytes, kWsBytes = (size_t)kGroupsPerBlock * kGemmM * 4;
constexpr size_t kXsOff = kWsOff + kWsBytes, kXsBytes = (size_t)kGroupsPerBlock * kGemmN * 4;
constexpr size_t kBarOff = kXsOff + kXsBytes;
constexpr size_t kGemmSmem = kBarOff + 64;
// Over half of the SM's shared memory, so one CTA per SM: a second CTA's 512-column TMEM allocation
// would wait for the first to free its columns.
constexpr size_t kGemmSmemLaunch = 120 * 1024;
static_assert(kGemmSmem <= kGemmSmemLaunch, "gemm shared memory");

// Canonical K-major, no-swizzle operand tile of R rows x 32 bytes: core matrices of 8 rows x 16 bytes
// (128 contiguous bytes); the R/8 row groups 128 bytes apart (SBO), the two 16-byte K halves R*16
// bytes apart (LBO).
__device__ __forceinline__ uint32_t core_off(int row, int half, int rows) {
    return (uint32_t)((row >> 3) * 128 + (row & 7) * 16 + half * rows * 16);
}
// tcgen05 shared-memory matrix descriptor (no swizzle, sm_100 version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: s32 accumulator, signed int8 A and B, both K-major, M x N.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGemmN >> 3) << 17) |
                            ((uint32_t)(kGemmM >> 4) << 24);

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar_smem) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_smem)
                 : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_q8_kernel(const GemmArgs g) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n = g.n, d = g.d, T = g.T;
    const int t0 = blockIdx.x * kGemmN, r0 = blockIdx.y * kGemmM;
    const int row = r0 + tid;
    uint8_t *A = smem + kAOff, *B = smem + kBOff;
    float *ws_s = reinterpret_cast<float *>(smem + kWsOff), *xs_s = reinterpret_cast<float *>(smem + kXsOff);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kBarOff);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + kBarOff + 16);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + kBarOff + 24);

    if (warp == 0) {
        tmem_alloc(smem_u32(tslot), kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        *abort = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    float sum[kGemmN];
    #pragma unroll
    for (int t = 0; t < kGemmN; ++t) sum[t] = 0.0f;
    const int nblk = (n + 511) >> 9;
    for (int b = 0; b < nblk; ++b) {
        const int wb = q8_blk_width(n, b), ng = wb >> 5;
        // ---- stage the block: weight rows (de-swizzled from the packed segments) and token values
        {
            const uint8_t *seg = row < d ? g.w + q8_seg_off(n, T, row, b) : nullptr;
            const int r = row % T;
            for (int c = 0; c < 2 * ng; ++c) {
                uint4 v = make_uint4(0, 0, 0, 0);
                if (seg) v = __ldg(reinterpret_cast<const uint4 *>(seg + 16 * q8_swz_q(c, r, wb)));
                *reinterpret_cast<uint4 *>(A + (size_t)(c >> 1) * kGemmM * 32 + core_off(tid, c & 1, kGemmM)) = v;
            }
            for (int k = 0; k < ng; ++k)
                ws_s[k * kGemmM + tid] =
                    seg ? __ldg(reinterpret_cast<const float *>(seg + wb + 16 * q8_swz_s(k >> 2, r, wb) + 4 * (k & 3)))
                        : 0.0f;
        }
        for (int i = tid; i < kGemmN * 2 * ng; i += kGemmThreads) {
            const int t = i / (2 * ng), c = i % (2 * ng);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (t0 + t < g.ntok) v = __ldg(reinterpret_cast<const uint4 *>(g.xq + (size_t)(t0 + t) * n + 512 * b + 16 * c));
            *reinterpret_cast<uint4 *>(B + (size_t)(c >> 1) * kGemmN * 32 + core_off(t, c & 1, kGemmN)) = v;
        }
        for (int i = tid; i < kGemmN * ng; i += kGemmThreads) {
            const int t = i / ng, k = i % ng;
            xs_s[k * kGemmN + t] = t0 + t < g.ntok ? __ldg(g.xs + (size_t)(t0 + t) * (n / 32) + 16 * b + k) : 0.0f;
        }
        fence_proxy_async_smem();  // the generic-proxy stores above, before the tensor cores read them
        tc_fence_before();
        __syncthreads();
        // ---- one MMA per group, each into its own accumulator
        if (tid == 0) {
            tc_fence_after();
            for (int k = 0; k < ng; ++k) {
                const uint64_t ad = smem_desc(smem_u32(A + (size_t)k * kGemmM * 32), kGemmM * 16, 128);
                const uint64_t bd = smem_desc(smem_u32(B + (size_t)k * kGemmN * 32), kGemmN * 16, 128);
                mma_i8(tmem + (uint32_t)(k * kGemmN), ad, bd);
            }
            mma_commit(smem_u32(bar));
        }
        // ---- fold the group terms in order
        if (!mbar_wait(bar, (uint32_t)(b & 1), g.err)) *abort = 1;
        tc_fence_after();
        if (!*abort) {
            for (int k = 0; k < ng; ++k) {
                int32_t dot[kGemmN];
                tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(k * kGemmN), dot);
                tmem_wait_ld();
                const float wsk = ws_s[k * kGemmM + tid];
                #pragma unroll
                for (int t = 0; t < kGemmN; ++t)
                    sum[t] = __fadd_rn(sum[t], __fmul_rn(__int2float_rn(dot[t]), __fmul_rn(wsk, xs_s[k * kGemmN + t])));
            }
        }
        tc_fence_before();
        __syncthreads();  // TMEM read and shared memory free before the next block overwrites them
        if (*abort) break;
    }
    // ---- epilogue
    if (!*abort) {
        if (g.epi == EPI_SWIGLU) {
            #pragma unroll
            for (int t = 0; t < kGemmN; ++t) {
                const float h3 = __shfl_down_sync(FULL, sum[t], 1);
                if (!(tid & 1) && row < d && t0 + t < g.ntok) {
                    // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                    const float v = __fmul_rn(sum[t], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-sum[t]))));
                    g.out[(size_t)(t0 + t) * (d >> 1) + (row >> 1)] = __fmul_rn(v, h3);
                }
            }
        } else if (row < d) {
            #pragma unroll
            for (int t = 0; t < kGemmN; ++t) {
                if (t0 + t >= g.ntok) break;
                float *o = g.out + (size_t)(t0 + t) * d + row;
                *o = g.epi == EPI_ADD ? __fadd_rn(*o, sum[t]) : sum[t];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

bool gemm_supported(int n, int d, int ntok, int epi) {
    return n > 0 && n % 32 == 0 && d > 0 && ntok > 0 && (epi == EPI_STORE || epi == EPI_ADD || (epi == EPI_SWIGLU && d % 2 == 0));
}

cudaError_t launch_gemm(const GemmArgs &g, cudaStream_t st) {
    if (!gemm_supported(g.n, g.d, g.ntok, g.epi) || g.T < 1 || g.T > 32) return cudaErrorInvalidValue;
    static int attr_set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmemLaunch);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    // token tiles along x: the CTAs of one row tile run side by side and share its weight reads in L2
    dim3 grid((g.ntok + kGemmN - 1) / kGemmN, (g.d + kGemmM - 1) / kGemmM);
    if (grid.y > 65535) return cudaErrorInvalidValue;
    gemm_q8_kernel<<<grid, kGemmThreads, kGemmSmemLaunch, st>>>(g);
    return cudaGetLastError();
}

}  // namespace dk
