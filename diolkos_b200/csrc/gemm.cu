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
#include <cstdlib>
#include <cstring>

#include <cuda.h>  // CUtensorMap and its enums; the encoder is fetched from the driver at run time

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


// ================================================================================================
// The pipelined form (n a multiple of 128, packed tiles of 17..32 rows): TMA + warp specialisation.
//
// The packed layout already is the tensor cores' 128-byte-swizzled K-major layout, one 128-value
// quarter of a block at a time: chunk c of tile row r sits at 16-byte position c ^ (r & 7) of its
// quarter, which is where the SWIZZLE_128B pattern puts it when row r of the tile is row r (mod 8) of
// an 8-row atom.  So TMA copies the packed bytes as they are (no swizzle of its own): per quarter, one
// 4-D box [128 B][32 rows][1 block][4 tiles] lands as 128 rows x 128 B, tile j at rows 32j..32j+31 (rows
// past the tile height T read as zeros); the matrix descriptor reads it with SWIZZLE_128B, SBO 1 KB,
// advancing 32 B per group.  The activations are a plain 2-D int8 map swizzled by TMA the same way.
//
// CTA = 4 packed tiles (128 rows) x 64 tokens, 18 warps:
//   warp 0   one thread issues the TMA copies of each 512-column block into a 2-stage ring;
//   warp 1   allocates TMEM; one thread issues one MMA per group (K = 32, s32) into a ring of 8
//            64-column TMEM accumulators and commits each to its mbarrier;
//   warps 2-17 fold: warp w reads the lanes of tile w % 4 (row = lane) and 16 of the 64 token columns
//            (the next group's columns load while the current one folds), refills the read columns
//            with the bias below and hands them back, and adds term = (float)dot * (ws * xs) to its
//            running sums in group order, the GEMV's arithmetic.
//            (float)dot is exact: the accumulators start at the bits 0x4B400000 and
//            |dot| <= 32 * 128 * 128 < 2^22, so the s32 sum's bits are the float 1.5 * 2^23 + dot, and
//            subtracting 1.5 * 2^23 is exact.
// Every wait is bounded and gives up when another role has; TMEM is always freed.
constexpr int kTcM = 128, kTcN = 64, kTcThreads = 576, kTcEpiWarps = 16, kTcTiles = 4, kTcTileRows = 32;
constexpr uint32_t kTcSlots = 8, kTcSlotCols = 64, kTcTmemCols = kTcSlots * kTcSlotCols;
// one stage: A [4 quarters][128 rows][128 B] | B [4 quarters][64 tokens][128 B] | weight scales [128 rows][64 B]
// | activation scales [64 tokens][16] | the same transposed [16][64]
constexpr size_t kStA = 0, kStB = 65536, kStWs = 98304, kStXs = 106496, kStXt = 110592, kStBytes = 114688;
constexpr int kTcStages = 2;
constexpr size_t kTcBarOff = kTcStages * kStBytes;
constexpr size_t kTcSmem = kTcBarOff + 256 + 1024;  // barriers, then slack to align the base to 1 KB
static_assert(kTcSmem <= 227 * 1024, "gemm stages");
constexpr uint32_t kIdescTc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(kTcM >> 4) << 24);

struct GemmMaps {
    CUtensorMap a[4];       // full blocks, quarter Q of the values: [128 B][T rows][blocks][tiles]
    CUtensorMap s;          // full blocks, the scale chunks: [64 B][T][blocks][tiles]
    CUtensorMap a_last[3];  // the last block when it is narrower (w % 128 == 0): [128 B][T][tiles]
    CUtensorMap s_last;     // [w/8 B][T][tiles]
    CUtensorMap x;          // activations int8 [ntok][n], box [128 B][64 tokens], 128-byte swizzle
    CUtensorMap xs;         // activation scales fp32 [ntok][n/32], box [16][64]
};
struct GemmTmaParams {
    GemmArgs g;
    GemmMaps m;
    int nfull;    // full 512-column blocks
    int wb_last;  // width of the narrower last block (0: none)
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
                   "r"(smem_u32(bar))
                 : "memory");
}
// Matrix descriptor of a 128-byte-swizzled K-major operand: 8-row atoms of 128-byte rows, atoms 1 KB apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
__device__ __forceinline__ void mma_i8_tc(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdescTc), "r"(1)
        : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane, and the wait that makes them usable (the
// registers are operands of the wait, so no use of them is scheduled before it).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld16(int32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
                 :
                 : "memory");
}
__device__ __forceinline__ void gemm_mark(const GemmArgs &g, int b, int k) {
    const int cta = blockIdx.y * gridDim.x + blockIdx.x;
    if (g.trace && cta < g.trace_ctas && b < g.trace_blocks) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g.trace[((size_t)cta * g.trace_blocks + b) * kGemmTraceSlots + k] = t;
    }
}
// 16 consecutive TMEM columns of this thread's lane set to v; the wait makes the store complete.
__device__ __forceinline__ void tmem_st16_fill(uint32_t taddr, uint32_t v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 "
                 "[%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(v)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Fold one group into 16 running sums: term = (float)dot * (ws * xs[t]), added in group order.  The
// accumulator columns hold the float 1.5 * 2^23 + dot.
__device__ __forceinline__ void fold_group(float (&sum)[16], const int32_t (&d)[16], float ws, const float *xq) {
    const float4 *xq4 = reinterpret_cast<const float4 *>(xq);
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 x4 = xq4[i];
        const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
        #pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float f = __fsub_rn(__int_as_float(d[4 * i + c]), 12582912.0f);
            sum[4 * i + c] = __fadd_rn(sum[4 * i + c], __fmul_rn(f, __fmul_rn(ws, xv[c])));
        }
    }
}
__device__ __forceinline__ void bar_epi() {  // the fold warps
    asm volatile("bar.sync 1, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_q8_tma_kernel(const __grid_constant__ GemmTmaParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const GemmArgs &g = P.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kTcN, tile0 = blockIdx.y * kTcTiles;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kTcBarOff);  // [2]
    uint64_t *empty = full + kTcStages;                                 // [2]
    uint64_t *tfull = empty + kTcStages;                                // [8]
    uint64_t *tempty = tfull + kTcSlots;                                // [8]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + kTcSlots);
    int *abort = reinterpret_cast<int *>(tslot + 1);
    const int nblk = P.nfull + (P.wb_last ? 1 : 0);

    if (warp == 1) {
        tmem_alloc(smem_u32(tslot), kTcTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kTcEpiWarps);
        }
        for (uint32_t k = 0; k < kTcSlots; ++k) {
            mbar_init(&tfull[k], 1);
            mbar_init(&tempty[k], kTcEpiWarps);
        }
        *abort = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            int issued[kTcStages] = {-1, -1};
            for (int b = 0; b < nblk; ++b) {
                const int s = b & 1;
                if (b >= kTcStages && !mbar_wait_abortable(&empty[s], (uint32_t)(((b >> 1) - 1) & 1), g.err, abort, false)) {
                    *abort = 1;
                    break;
                }
                const bool part = b == P.nfull;
                const int wb = part ? P.wb_last : 512, nq = wb >> 7;
                uint8_t *st = smem + (size_t)s * kStBytes;
                mbar_arrive_expect_tx(&full[s], (uint32_t)(nq * (16384 + 8192) + (wb / 8) * kTcM + 4096));
                for (int q = 0; q < nq; ++q) {
                    if (!part) tma_load_4d(st + kStA + q * 16384, &P.m.a[q], 0, 0, b, tile0, &full[s]);
                    else tma_load_3d(st + kStA + q * 16384, &P.m.a_last[q], 0, 0, tile0, &full[s]);
                    tma_load_2d(st + kStB + q * 8192, &P.m.x, 512 * b + 128 * q, t0, &full[s]);
                }
                if (!part) tma_load_4d(st + kStWs, &P.m.s, 0, 0, b, tile0, &full[s]);
                else tma_load_3d(st + kStWs, &P.m.s_last, 0, 0, tile0, &full[s]);
                tma_load_2d(st + kStXs, &P.m.xs, 16 * b, t0, &full[s]);
                issued[s] = b;
                gemm_mark(g, b, 0);
            }
            // never leave with copies still landing in shared memory
            for (int s = 0; s < kTcStages; ++s)
                if (issued[s] >= 0) mbar_wait(&full[s], (uint32_t)((issued[s] >> 1) & 1), g.err);
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            uint32_t gseq = 0;
            int last_k = -1;
            uint32_t last_par = 0;
            bool ok = true;
            for (int b = 0; b < nblk && ok; ++b) {
                const int s = b & 1;
                if (!mbar_wait_abortable(&full[s], (uint32_t)((b >> 1) & 1), g.err, abort, false)) {
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                gemm_mark(g, b, 1);
                const int ng = (b == P.nfull ? P.wb_last : 512) >> 5;
                const uint32_t a0 = smem_u32(smem + (size_t)s * kStBytes + kStA);
                const uint32_t b0 = smem_u32(smem + (size_t)s * kStBytes + kStB);
                for (int q = 0; q < ng; ++q, ++gseq) {
                    const uint32_t k = gseq & (kTcSlots - 1);
                    // the slot holds the bias again (stored by the fold warps: first at the start, then
                    // each time they have read it)
                    if (!mbar_wait_abortable(&tempty[k], (gseq / kTcSlots) & 1, g.err, abort, false)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_i8_tc(tmem + k * kTcSlotCols, sw128_desc(a0 + (q >> 2) * 16384 + (q & 3) * 32),
                              sw128_desc(b0 + (q >> 2) * 8192 + (q & 3) * 32));
                    mma_commit(smem_u32(&tfull[k]));
                    last_k = (int)k;
                    last_par = (gseq / kTcSlots) & 1;
                }
                if (ok) mma_commit(smem_u32(&empty[s]));
                gemm_mark(g, b, 2);
            }
            // the tensor cores are done with TMEM before it is freed
            if (last_k >= 0) mbar_wait(&tfull[last_k], last_par, g.err);
        }
    } else {
        // ---- fold warps: warp w reads the lanes of tile w % 4 and the 16 token columns 16 * ((w - 2) / 4) ..
        // The accumulators start at the bias 0x4B400000 (the float 1.5 * 2^23): the MMA adds the s32 dot,
        // so each column holds the float 1.5 * 2^23 + dot and (float)dot is one exact subtraction.
        const int lq = warp & 3, h = (warp - 2) >> 2, et = tid - 64;
        const int T = g.T, r = lane, row = (tile0 + lq) * T + r;
        const int tok0 = t0 + 16 * h;
        const bool any_tok = tok0 < g.ntok;
        const uint32_t tbase = tmem + ((uint32_t)(32 * lq) << 16) + 16 * h;
        constexpr uint32_t kBias = 0x4B400000u;
        float sum[16];
        #pragma unroll
        for (int t = 0; t < 16; ++t) sum[t] = 0.0f;
        bool ok = true;
        // A slot read into registers is refilled with the bias; it goes back to the MMA thread at the next
        // release (or flush), once the store is known complete, so the store's latency is not waited on.
        int pending = -1;
        auto flush = [&]() {
            if (pending < 0) return;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[pending]);
            pending = -1;
        };
        auto release = [&](uint32_t gq) {
            flush();
            tmem_st16_fill(tbase + (gq & (kTcSlots - 1)) * kTcSlotCols, kBias);
            pending = (int)(gq & (kTcSlots - 1));
        };
        for (uint32_t k = 0; k < kTcSlots; ++k) release(k);  // first fill of every slot
        flush();
        // bounded wait for group gq's accumulator, the same outcome on every lane
        auto wait_acc = [&](uint32_t gq) {
            const bool got = mbar_wait_abortable(&tfull[gq & (kTcSlots - 1)], (gq / kTcSlots) & 1, g.err, abort, false);
            if (!__all_sync(FULL, got)) {
                *abort = 1;
                ok = false;
            }
            if (ok) tc_fence_after();
            return ok;
        };
        auto load_acc = [&](uint32_t gq, int32_t(&d)[16]) {
            tmem_ld16(tbase + (gq & (kTcSlots - 1)) * kTcSlotCols, d);
        };
        uint32_t gseq = 0;
        // every fold warp passes the per-block barrier once per block, whatever happened before
        for (int b = 0; b < nblk; ++b) {
            const int s = b & 1;
            if (ok) {
                const bool got = mbar_wait_abortable(&full[s], (uint32_t)((b >> 1) & 1), g.err, abort, false);
                ok = __all_sync(FULL, got);
                if (!ok) *abort = 1;
            }
            if (warp == 2 && lane == 0) gemm_mark(g, b, 3);
            const uint8_t *st = smem + (size_t)s * kStBytes;
            const int wb = b == P.nfull ? P.wb_last : 512, ng = wb >> 5;
            // the activation scales transposed to [group][token] (2 per thread), then every fold warp
            float *xt = reinterpret_cast<float *>(const_cast<uint8_t *>(st) + kStXt);
            if (ok) {
                const float *xsm = reinterpret_cast<const float *>(st + kStXs);
                #pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int e = et + i * kTcEpiWarps * 32, tk = e >> 4, gg = e & 15;
                    xt[gg * kTcN + tk] = xsm[e];
                }
            }
            bar_epi();
            if (__any_sync(FULL, *reinterpret_cast<volatile int *>(abort) != 0)) ok = false;
            if (ok) {
                // this row's weight scales: scale q at chunk q8_swz_s(q / 4), word q % 4
                const uint8_t *wsr = st + kStWs + (size_t)(32 * lq + r) * (wb / 8);
                const float *xth = xt + 16 * h;
                auto scale = [&](int q) {
                    return *reinterpret_cast<const float *>(wsr + 16 * q8_swz_s(q >> 2, r, wb) + 4 * (q & 3));
                };
                // group q+1's accumulator loads while group q folds (two register sets, groups in pairs)
                int32_t da[16], db[16];
                if (wait_acc(gseq)) {
                    if (any_tok) {
                        load_acc(gseq, da);
                        tmem_wait_ld16(da);
                    }
                    release(gseq);
                }
                for (int q = 0; ok && q < ng; q += 2) {  // ng is a multiple of 4
                    const uint32_t g1 = gseq + q + 1, g2 = gseq + q + 2;
                    if (!wait_acc(g1)) break;
                    if (any_tok) load_acc(g1, db);
                    if (any_tok) fold_group(sum, da, scale(q), xth + q * kTcN);
                    if (any_tok) tmem_wait_ld16(db);
                    release(g1);
                    const bool more = q + 2 < ng;
                    if (more) {
                        if (!wait_acc(g2)) break;
                        if (any_tok) load_acc(g2, da);
                    }
                    if (any_tok) fold_group(sum, db, scale(q + 1), xth + (q + 1) * kTcN);
                    if (more) {
                        if (any_tok) tmem_wait_ld16(da);
                        release(g2);
                    }
                }
            }
            gseq += ng;
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&empty[s]);
            if (warp == 2 && lane == 0) gemm_mark(g, b, 4);
        }
        flush();
        // epilogue: this thread's row, 16 tokens
        if (ok && any_tok) {
            const bool live = r < T && row < g.d;
            if (g.epi == EPI_SWIGLU) {
                #pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const float h3 = __shfl_down_sync(FULL, sum[t], 1);
                    if (live && !(r & 1) && tok0 + t < g.ntok) {
                        // val *= 1/(1+expf(-val)); val *= hb2 (src/transformer.c:214-220)
                        const float v = __fmul_rn(sum[t], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-sum[t]))));
                        g.out[(size_t)(tok0 + t) * (g.d >> 1) + (row >> 1)] = __fmul_rn(v, h3);
                    }
                }
            } else if (live) {
                #pragma unroll
                for (int t = 0; t < 16; ++t) {
                    if (tok0 + t >= g.ntok) break;
                    float *o = g.out + (size_t)(tok0 + t) * g.d + row;
                    *o = g.epi == EPI_ADD ? __fadd_rn(*o, sum[t]) : sum[t];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcTmemCols);
    }
}

}  // namespace

bool gemm_supported(int n, int d, int ntok, int epi) {
    return n > 0 && n % 32 == 0 && d > 0 && ntok > 0 && (epi == EPI_STORE || epi == EPI_ADD || (epi == EPI_SWIGLU && d % 2 == 0));
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool encode(CUtensorMap *m, CUtensorMapDataType type, int rank, const void *base, const cuuint64_t *dims,
            const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle swz) {
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return encode_fn()(m, type, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor maps of the pipelined form; false when a shape or address does not fit it.
bool make_maps(const GemmArgs &g, GemmTmaParams &P) {
    const int n = g.n, T = g.T;
    if (n % 128 || T <= 16 || T > kTcTileRows || !encode_fn()) return false;
    if ((reinterpret_cast<uintptr_t>(g.w) | reinterpret_cast<uintptr_t>(g.xq) | reinterpret_cast<uintptr_t>(g.xs)) & 15)
        return false;
    const int ntiles = (g.d + T - 1) / T;
    const uint64_t rowb = q8_row_bytes(n), tileb = (uint64_t)T * rowb;
    P.g = g;
    P.nfull = n / 512;
    P.wb_last = n % 512;
    const uint8_t *w = g.w;
    if (P.nfull > 0) {
        for (int q = 0; q < 4; ++q) {
            const cuuint64_t dims[4] = {128, (cuuint64_t)T, (cuuint64_t)P.nfull, (cuuint64_t)ntiles};
            const cuuint64_t str[3] = {576, (cuuint64_t)T * 576, tileb};
            const cuuint32_t box[4] = {128, kTcTileRows, 1, kTcTiles};
            if (!encode(&P.m.a[q], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w + 128 * q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
                return false;
        }
        const cuuint64_t dims[4] = {64, (cuuint64_t)T, (cuuint64_t)P.nfull, (cuuint64_t)ntiles};
        const cuuint64_t str[3] = {576, (cuuint64_t)T * 576, tileb};
        const cuuint32_t box[4] = {64, kTcTileRows, 1, kTcTiles};
        if (!encode(&P.m.s, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w + 512, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    if (P.wb_last) {
        const int wb = P.wb_last;
        const uint64_t blk = q8_blk_bytes(wb);
        const uint8_t *base = w + (size_t)P.nfull * T * 576;
        for (int q = 0; q < wb / 128; ++q) {
            const cuuint64_t dims[3] = {128, (cuuint64_t)T, (cuuint64_t)ntiles};
            const cuuint64_t str[2] = {blk, tileb};
            const cuuint32_t box[3] = {128, kTcTileRows, kTcTiles};
            if (!encode(&P.m.a_last[q], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + 128 * q, dims, str, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE))
                return false;
        }
        const cuuint64_t dims[3] = {(cuuint64_t)(wb / 8), (cuuint64_t)T, (cuuint64_t)ntiles};
        const cuuint64_t str[2] = {blk, tileb};
        const cuuint32_t box[3] = {(cuuint32_t)(wb / 8), kTcTileRows, kTcTiles};
        if (!encode(&P.m.s_last, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + wb, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)g.ntok};
        const cuuint64_t str[1] = {(cuuint64_t)n};
        const cuuint32_t box[2] = {128, kTcN};
        if (!encode(&P.m.x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, g.xq, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(n / 32), (cuuint64_t)g.ntok};
        const cuuint64_t str[1] = {(cuuint64_t)(n / 32) * 4};
        const cuuint32_t box[2] = {16, kTcN};
        if (!encode(&P.m.xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, g.xs, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    return true;
}

}  // namespace

// DIOLKOS_GEMM_TRACE=1: the pipelined form records the first 148 CTAs' first 32 blocks (dk_gemm_trace).
static unsigned long long *g_trace = nullptr;
static constexpr int kTraceCtas = 148, kTraceBlocks = 32;

unsigned long long *gemm_trace_buffer(int *ctas, int *blocks) {
    *ctas = kTraceCtas;
    *blocks = kTraceBlocks;
    return g_trace;
}

bool gemm_pipelined(const GemmArgs &g) {
    GemmTmaParams P;
    return gemm_supported(g.n, g.d, g.ntok, g.epi) && make_maps(g, P);
}

cudaError_t launch_gemm(const GemmArgs &g, cudaStream_t st) {
    if (!gemm_supported(g.n, g.d, g.ntok, g.epi) || g.T < 1 || g.T > 32) return cudaErrorInvalidValue;
    static int attr_set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmemLaunch);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_q8_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    static const bool simple_only = [] {  // DIOLKOS_GEMM=simple: the simple form for every shape
        const char *e = getenv("DIOLKOS_GEMM");
        return e && strcmp(e, "simple") == 0;
    }();
    static const bool tracing = [] {
        const char *e = getenv("DIOLKOS_GEMM_TRACE");
        return e && atoi(e) > 0;
    }();
    GemmTmaParams P;
    if (!simple_only && make_maps(g, P)) {
        if (tracing) {
            if (!g_trace &&
                cudaMalloc(&g_trace, sizeof(unsigned long long) * kTraceCtas * kTraceBlocks * kGemmTraceSlots) != cudaSuccess)
                return cudaErrorMemoryAllocation;
            P.g.trace = g_trace;
            P.g.trace_ctas = kTraceCtas;
            P.g.trace_blocks = kTraceBlocks;
        }
        const int ntiles = (g.d + g.T - 1) / g.T;
        dim3 grid((g.ntok + kTcN - 1) / kTcN, (ntiles + kTcTiles - 1) / kTcTiles);
        if (grid.y > 65535) return cudaErrorInvalidValue;
        gemm_q8_tma_kernel<<<grid, kTcThreads, kTcSmem, st>>>(P);
        return cudaGetLastError();
    }
    // token tiles along x: the CTAs of one row tile run side by side and share its weight reads in L2
    dim3 grid((g.ntok + kGemmN - 1) / kGemmN, (g.d + kGemmM - 1) / kGemmM);
    if (grid.y > 65535) return cudaErrorInvalidValue;
    gemm_q8_kernel<<<grid, kGemmThreads, kGemmSmemLaunch, st>>>(g);
    return cudaGetLastError();
}

}  // namespace dk
