// dk_kernels.h -- host-side launch interface of the Diolkos B200 kernels (internal to the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dk {

// ---------------- GEMV -----------------------------------------------------------------------
// Activation prologue: how the CTA builds the Q8_0 activation in shared memory.
enum GemvPro : int {
    PRO_Q8 = 0,       // already quantised: xq int8[n], xs fp32[n/32]
    PRO_F32 = 1,      // quantise fp32 x[n] (convert_f32_q8, src/tensor.c:199)
    PRO_RMS = 2,      // rmsnorm(x, norm_w) then quantise (src/utils.c:59 + src/tensor.c:199)
    PRO_EMB_RMS = 3,  // x = dequant(embedding row tokens[*pos]) (written back by CTA 0), then as PRO_RMS
    PRO_RMS_REDUCE = 4,  // tensor parallel: wait for every rank's partial rows, x_out = x + sum over ranks
                         // (rank order; written by CTA 0), then as PRO_RMS on x_out
};
// Epilogue: what happens to each finished row value.
enum GemvEpi : int {
    EPI_STORE = 0,   // out[row] = v
    EPI_ADD = 1,     // out[row] += v (residual, src/transformer.c:199-201, :228-230)
    EPI_SWIGLU = 2,  // rows (2i, 2i+1) = (w1_i, w3_i): out[i] = silu(v0) * v1 (src/transformer.c:212-222)
    EPI_ARGMAX = 3,  // out[row] = v, and the greedy token (src/sampler.c:6-17) is written to tokens[pos+1]
    EPI_NONE = 4,    // partial sums only (tensor-parallel split: the caller reduces)
    EPI_PEER = 5,    // tensor parallel: store each row's partial sum into every rank's receive area
                     // (over NVLink peer memory), then count the rows on every rank's counter
};

struct GemvArgs {
    const uint8_t *w = nullptr;  // packed matrix (tile layout)
    int n = 0, d = 0;
    int pro = PRO_F32, epi = EPI_STORE;
    const float *x = nullptr;       // PRO_F32 / PRO_RMS input; PRO_EMB_RMS: x is written here
    const float *norm_w = nullptr;  // PRO_RMS / PRO_EMB_RMS
    const int8_t *xq = nullptr;     // PRO_Q8
    const float *xs = nullptr;
    const uint8_t *emb = nullptr;   // PRO_EMB_RMS: packed embedding table
    int emb_T = 32;                 // its tile height
    float *out = nullptr;
    // greedy-token epilogue and embedding prologue state (device memory)
    unsigned long long *amax_part = nullptr;  // >= grid entries
    unsigned int *amax_count = nullptr;       // zero between launches
    int *tokens = nullptr;                    // token buffer (capacity >= seq_len + 1)
    int *pos = nullptr;                       // current position (incremented by EPI_ARGMAX)
    const int *n_forced = nullptr;            // prompt length: tokens[0..n_forced) are forced
    int seq_len = 0;
    int *err = nullptr;                       // device error word
    // ---- tensor-parallel exchange (tp_world > 1) ----
    int tp_rank = 0, tp_world = 1;
    // EPI_PEER: [tp_world] device pointers to each rank's receive area for this exchange point
    // (float[tp_world][d], indexed by the source rank) and to each rank's counter for it.
    float *const *peer_recv = nullptr;
    unsigned long long *const *peer_cnt = nullptr;
    // PRO_RMS_REDUCE: this rank's receive area (float[tp_world][n]) and counter; the wait ends when the
    // counter reaches (epoch * red_period + red_index + 1) * tp_world * n.
    const float *recv = nullptr;
    const unsigned long long *cnt = nullptr;
    int red_index = 0, red_period = 0;
    const unsigned long long *epoch = nullptr;  // decode steps completed (advanced by the classifier)
    float *x_out = nullptr;
    // EPI_ARGMAX across ranks: each rank's key array (u64[tp_world]) and its counter; this rank's own.
    unsigned long long *const *peer_amax = nullptr;
    unsigned long long *const *peer_amax_cnt = nullptr;
    const unsigned long long *amax_keys = nullptr;
    const unsigned long long *amax_keys_cnt = nullptr;
    unsigned long long *epoch_rw = nullptr;     // the classifier's writable view of epoch
    int row_offset = 0;                         // global index of this rank's first classifier row
    int vocab = 0;                              // rows of the whole classifier (0: d)
    // ---- tensor parallel, persistent step: the tagged exchange (tagged != 0) ----
    // Partial rows and the residual travel as 64-bit words, (tag << 32) | value bits, so that a reader
    // tells a new value from an old one by the word alone: no fences and no counters.  The tag of event k
    // of a step (k = 0: the embedding row, k = 2l+1: the reduce after layer l's wo, k = 2l+2: after its w2)
    // is epoch * tag_period + k + 1 (tag_period = 2 * layers + 1).
    //   EPI_PEER:       each row's partial sum into every rank's peer_recv64[q][tp_rank * d + row], tag k;
    //   PRO_RMS_REDUCE: gatherer CTAs 0 .. n_gather-1 each take a slice of the rows: wait for every rank's
    //                   partial (recv64[q][row], tag k) and the residual (x64[row], tag k-1), sum in rank
    //                   order and store x64_out[row] (tag k); then every CTA reads x64_out (tag k);
    //   PRO_EMB_RMS:    the CTA that owns tile 0 stores the embedding row to x64_out (tag 0).
    int tagged = 0, n_gather = 0;
    int tag_k = 0, tag_period = 0;
    const unsigned long long *x64 = nullptr;
    unsigned long long *x64_out = nullptr;
    const unsigned long long *recv64 = nullptr;
    unsigned long long *const *peer_recv64 = nullptr;
    // Standalone kernel, PRO_F32 / EPI_STORE only: the input x was complete before the previous kernel in
    // the stream started (the later GEMVs of dk_matmul_q8_0_batch, whose first GEMV is launched without
    // programmatic dependence), so the activation is built and the terms computed before the dependency
    // wait, which only the output stores take.
    int early_input = 0;
    // Diagnostics (persistent step only; nullptr: off): the CTA that owns tile 0 copies the op's fp32
    // input vector (n floats; the residual written by the prologue where it writes one) and the Q8_0
    // activation it built (n int8, n/32 scales) here, for per-layer parity checks.
    float *dump_in = nullptr;
    int8_t *dump_q = nullptr;
    float *dump_s = nullptr;
};

struct GemvPlan {
    int T = 32;        // rows per tile (the packed layout's tile height)
    int ntiles = 0;    // tiles of the matrix
    int grid = 1;      // CTAs (one contiguous tile range each)
    int NW = 1;        // consumer warps (stage s of the CTA goes to warp s % NW)
    int S = 1;         // ring slots (stage s of the CTA lands in slot s % S); S >= NW, S % NP == 0
    int NP = 1;        // producer threads (producer q issues the stages s = q mod NP)
    int PF = 0;        // stages prefetched into L2 ahead of the ring
    size_t slot = 0;   // bytes of one stage slot (T * 576)
    size_t xoff = 0;   // shared-memory offset of the activation
    size_t smem = 0;   // dynamic shared memory bytes
};

// ---- packed Q8_0 weight layout ----------------------------------------------------------------
// An n-column matrix is cut into 512-column blocks; block b holds w_b = min(512, n - 512b) columns
// and, per row, a SEGMENT of q8_blk_bytes(w_b) bytes: the row's w_b int8 values (16-byte chunks)
// followed by its w_b/32 fp32 scales, padded to 16 bytes (576 bytes for a full block).  Rows are
// grouped into tiles of T rows (T depends on the row count and the GPU's SM count so that every SM
// gets the same number of rows); a tile stores block 0 of its T rows, then block 1, ... so that
// (tile, block) -- one STAGE of the GEMV -- is one contiguous range of T segments.  Inside a
// segment the chunks are XOR-swizzled by the row's index in the tile so that lanes reading "their"
// rows hit distinct shared-memory banks.  The last tile is padded with zero rows.
__host__ __device__ inline int q8_blk_width(int n, int b) { return (n - 512 * b) < 512 ? (n - 512 * b) : 512; }
__host__ __device__ inline size_t q8_blk_bytes(int w) { return ((size_t)w + (size_t)w / 8 + 15) & ~(size_t)15; }
// Bytes of all segments of one row.
__host__ __device__ inline size_t q8_row_bytes(int n) {
    return (size_t)(n / 512) * 576 + ((n % 512) ? q8_blk_bytes(n % 512) : 0);
}
// Tile height for a d-row matrix on num_sms SMs (unit = 2 keeps SwiGLU row pairs in one tile).
__host__ __device__ inline int q8_tile_rows(int d, int num_sms, int unit) {
    const long per = 32L * num_sms;
    const long k = (d + per - 1) / per;  // tiles per SM
    long t = (d + (long)num_sms * k - 1) / ((long)num_sms * k);
    t = (t + unit - 1) / unit * unit;
    return (int)(t < 1 ? 1 : (t > 32 ? 32 : t));
}
__host__ __device__ inline size_t q8_packed_bytes(int n, int d, int T) {
    return (size_t)((d + T - 1) / T) * (size_t)T * q8_row_bytes(n);
}
// Byte offset of the segment (row, block b).
__host__ __device__ inline size_t q8_seg_off(int n, int T, int row, int b) {
    return (size_t)(row / T) * (size_t)T * q8_row_bytes(n) + (size_t)T * 576 * b +
           (size_t)(row % T) * q8_blk_bytes(q8_blk_width(n, b));
}
// Physical 16-byte position of value chunk c / scale chunk s in the segment of tile row r.
__host__ __device__ inline int q8_swz_q(int c, int r, int wb) { return ((wb / 16) % 8 == 0) ? (c ^ (r & 7)) : c; }
__host__ __device__ inline int q8_swz_s(int s, int r, int wb) {
    if (wb == 512) return s ^ ((r >> 1) & 3);
    if (wb == 256) return s ^ (r & 1);
    return s;
}
// The 32 dequantised values (q * scale) of group g of packed row `row`.
__host__ __device__ inline void q8_packed_group(const uint8_t *w, int n, int T, int row, int g, float *f) {
    const int b = g >> 4, wb = q8_blk_width(n, b), r = row % T, k = g & 15;
    const uint8_t *seg = w + q8_seg_off(n, T, row, b);
    const int8_t *c0 = reinterpret_cast<const int8_t *>(seg + 16 * q8_swz_q(2 * k, r, wb));
    const int8_t *c1 = reinterpret_cast<const int8_t *>(seg + 16 * q8_swz_q(2 * k + 1, r, wb));
    const float s = *reinterpret_cast<const float *>(seg + wb + 16 * q8_swz_s(k >> 2, r, wb) + 4 * (k & 3));
    for (int i = 0; i < 16; ++i) {
#ifdef __CUDA_ARCH__
        f[i] = __fmul_rn((float)c0[i], s);
        f[16 + i] = __fmul_rn((float)c1[i], s);
#else
        f[i] = (float)c0[i] * s;
        f[16 + i] = (float)c1[i] * s;
#endif
    }
}
size_t gemv_x_bytes(int n);
// Shared memory besides the ring: activation, reduction scratch, barriers, argmax keys.
size_t gemv_smem_tail(int n);
// Tile height of the matrix a GEMV with this epilogue runs on (d rows, num_sms SMs).
int gemv_tile_rows(int d, int epi, int num_sms);
GemvPlan plan_gemv(int n, int d, int epi, int num_sms);
bool gemv_supported(int n, int d, int epi);
cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl);
// A batch of same-shape matrices against one input in ONE launch (dk_matmul_q8_0_batch): every CTA
// streams its tiles of matrix 0, then of matrix 1, ... through one ring, the activation built once,
// out[i * d + row] for matrix i.  PRO_F32 or PRO_Q8 with EPI_STORE.
constexpr int kGemvBatchMax = 32;
struct GemvBatch {
    int count = 0;  // 0: the single matrix GemvArgs::w
    // CTA groups: group g (CTAs g * grid .. (g+1) * grid - 1 of the launch) takes matrices g, g + groups, ...
    // over the same tiles, so that `groups` CTAs share each SM, each with its own ring and row-sum chains
    int groups = 1;
    const uint8_t *w[kGemvBatchMax] = {};
};
GemvPlan plan_gemv_batch(int n, int d, int count, int num_sms);
cudaError_t launch_gemv_batch(const GemvArgs &a, const GemvBatch &b, const GemvPlan &p, cudaStream_t st, bool pdl);

// ---------------- batched Q8_0 matmul on the tensor cores (prefill) --------------------------
struct GemmArgs {
    const uint8_t *w = nullptr;  // packed matrix (tile layout, tile height T)
    int n = 0, d = 0, T = 32;
    const int8_t *xq = nullptr;  // activations: int8 [ntok][n], fp32 scales [ntok][n/32]
    const float *xs = nullptr;
    int ntok = 0;
    int epi = EPI_STORE;         // EPI_STORE: out[t][d]; EPI_ADD: out[t][d] +=; EPI_SWIGLU: out[t][d/2]
    float *out = nullptr;
    int *err = nullptr;
    // Optional timeline of the pipelined form (%globaltimer, ns), [CTA][block][kGemmTraceSlots]: producer
    // issued the block's copies, MMA thread saw them land, MMA thread issued its last group, fold warp 2
    // saw them land, fold warp 2 finished the block.
    unsigned long long *trace = nullptr;
    int trace_ctas = 0, trace_blocks = 0;
};
constexpr int kGemmTraceSlots = 5;
bool gemm_supported(int n, int d, int ntok, int epi);
cudaError_t launch_gemm(const GemmArgs &g, cudaStream_t st);
// The timeline buffer of the last traced launch (DIOLKOS_GEMM_TRACE=1), or nullptr.
unsigned long long *gemm_trace_buffer(int *ctas, int *blocks);

// ---------------- Q8_0 conversions ----------------------------------------------------------
cudaError_t launch_quant_bf16(const uint16_t *x, size_t n, int8_t *q, float *s, cudaStream_t st);
cudaError_t launch_quant_f16(const uint16_t *x, size_t n, int8_t *q, float *s, cudaStream_t st);
cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *q, float *s, cudaStream_t st);
cudaError_t launch_dequant(const int8_t *q, const float *s, size_t n, float *out, cudaStream_t st);
cudaError_t launch_group_dots(const int8_t *xq, const int8_t *wq, int n, int d, int32_t *dots, cudaStream_t st);
// Pack `rows` planar rows into packed rows row0, row0+step, ... of an n-column matrix with tile
// height T.  Source row i is columns [col0, col0+n) of a planar matrix with src_n columns: int8
// q[i*src_n + col0 ..], fp32 s[i*src_n/32 + col0/32 ..] (col0 % 32 == 0).  The destination must be
// zeroed beforehand (padding stays zero).
cudaError_t launch_pack_rows(uint8_t *dst, int n, int T, const int8_t *q, const float *s, int rows, int row0,
                             int step, cudaStream_t st, int src_n = 0, int col0 = 0);
cudaError_t launch_rmsnorm(float *o, const float *x, const float *w, int n, cudaStream_t st);
cudaError_t launch_embed(const uint8_t *emb_packed, int dim, int T, const int *tokens, const int *pos, float *x,
                         cudaStream_t st, bool pdl);

// ---------------- attention ------------------------------------------------------------------
// Smallest run of positions one attention CTA takes (splits are never shorter).
constexpr int kAttnMinChunk = 32;
// Split plan of the attention over T positions (0 .. T-1): nsplit runs of `chunk` positions, the last one
// shorter.  nsplit = min(max_splits, ceil(T / min_chunk)) rounds the chunk up; the split count then
// follows from the chunk, so that no split is empty (T = 385 over at most 24 splits: chunk 17, 23 splits).
__host__ __device__ inline void attn_split_plan(int T, int max_splits, int min_chunk, int &nsplit, int &chunk) {
    int n = (T + min_chunk - 1) / min_chunk;
    n = n < max_splits ? n : max_splits;
    n = n < 1 ? 1 : n;
    chunk = (T + n - 1) / n;
    nsplit = (T + chunk - 1) / chunk;
}
struct AttnArgs {
    const float *qkv = nullptr;  // [dim + 2*kv_dim]: q | k | v before RoPE
    const float *rope = nullptr; // [seq_len][head_size/2][2] (cos, sin)
    void *k_cache = nullptr;     // this layer: [n_kv_heads][seq_len][head_size], bf16 or f32
    void *v_cache = nullptr;
    float *out = nullptr;        // [n_heads*head_size]
    float *work = nullptr;       // split partials: [n_heads][max_splits][head_size + 2]
    unsigned int *count = nullptr; // [n_kv_heads] arrival counters (zero between launches)
    const int *pos = nullptr;
    int n_heads = 0, n_kv_heads = 0, head_size = 0, seq_len = 0;
    int kv_f32 = 0;
    // max_splits: the split capacity of `work` (its layout stride) and, for the standalone kernel, the cap of
    // its plan; min_chunk: that plan's shortest split.
    int max_splits = 1, min_chunk = kAttnMinChunk;
    // The persistent step's attention (and the prompt prefill's, which follows it) has two forms, chosen by
    // the number of positions T (step_attn_plan): up to wide_from positions, narrow items of
    // kAttnNarrowWarps warps over short splits (many items, a split merge); beyond, wide items on every
    // compute warp of a CTA over at most one wave of long splits.
    int narrow_max_splits = 1, narrow_min_chunk = 16;
    int wide_max_splits = 1, wide_min_chunk = 16;
    int wide_from = 0x7fffffff;
    int *err = nullptr;
};
constexpr int kAttnNarrowWarps = 2;   // warps of a narrow attention item
constexpr int kAttnWideWarps = 10;    // warps of a wide one: every compute warp of the persistent step's CTA
// The persistent step's attention form and split plan over T positions: returns the warps of an item.
__host__ __device__ inline int step_attn_plan(const AttnArgs &a, int T, int &nsplit, int &chunk) {
    if (T <= a.wide_from) {
        attn_split_plan(T, a.narrow_max_splits, a.narrow_min_chunk, nsplit, chunk);
        return kAttnNarrowWarps;
    }
    attn_split_plan(T, a.wide_max_splits, a.wide_min_chunk, nsplit, chunk);
    // A chunk rounded up to whole 8-position batches: an item's warps run the same batch rounds (a round
    // is 80 positions), and the chunk stays the same over runs of 8 x nsplit positions, so the prompt
    // prefill can group 8 positions per item.
    if (nsplit > 1) {
        chunk = (chunk + 7) & ~7;
        nsplit = (T + chunk - 1) / chunk;
        if (nsplit == 1) chunk = T;
    }
    return kAttnWideWarps;
}
int attn_max_splits(int seq_len, int n_kv_heads, int num_sms);
size_t attn_smem_bytes(const AttnArgs &a);
// Scratch of one attention launch: split partials (n_heads * max_splits * (head_size + 2) floats)
// at offset 0, then n_kv_heads arrival counters at attn_count_offset(); both 256-byte aligned.
size_t attn_count_offset(int n_heads, int head_size, int max_splits);
size_t attn_work_bytes(int n_heads, int n_kv_heads, int head_size, int max_splits);
// Shape checks of launch_attention (head_size a multiple of 4 and <= 128, n_heads a multiple of n_kv_heads
// with at most 8 query heads per KV head).
bool attn_supported(int n_heads, int n_kv_heads, int head_size);
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl);

// ---------------- persistent decode step ----------------------------------------------------------
// The whole step as one cooperative kernel (step.cu): a list of ops that every CTA walks in order.
constexpr int kStepProducers = 2;     // producer warps per CTA (one issuing thread each)
constexpr int kStepMaxSlots = 16;     // ring slots
constexpr int kStepMaxConsumers = 10; // GEMV consumer warps (at most the compute warps)
// Positions of the shortest split of the wide attention form (step_attn_plan): a wide item (one KV head, one
// split) runs on all compute warps of a CTA, 8 positions per warp per round, 80 per round.  A split takes up
// to 4 rounds (320 positions) before the plan cuts it -- a split merge costs two L2 round trips, a round
// about a third of one -- or fewer under grouped-query attention, where a round covers kv_mul query heads;
// never less than one round, so that no warp of an item idles (70B shape: 80 positions measured 2.6 % faster
// per token than 40, and 160 slower).
__host__ __device__ inline int step_min_chunk(int kv_mul) {
    const int c = 320 / (kv_mul > 0 ? kv_mul : 1);
    return c > 80 ? c : 80;
}
// Contexts up to this many positions take the narrow attention form (step_attn_plan), longer ones the wide
// (unless the wide items would leave more than a tenth of the CTAs idle; the engine then keeps the narrow
// form throughout).  Short contexts have too few positions to fill CTA-wide items.  Measured at 2048+
// positions on B200: the 70B shape (144 wide items on 148 SMs) 63.8 tok/s wide against 60.6 narrow; the 7B
// shape on 2 GPUs (144 items) 514 against 508; the 7B shape on one GPU (128 items) 388 against 396.
// Switching at 256, 384 or 640 positions measured the same on the 7B and 70B decode workloads.
constexpr int kStepWideFrom = 384;
enum StepOpKind : int { OP_GEMV = 0, OP_ATTN = 1 };
struct StepOp {
    int kind = OP_GEMV;
    GemvArgs g;             // OP_GEMV: matrix, prologue, epilogue (the standalone GEMV's arguments)
    int T = 32, ntiles = 0; // OP_GEMV: the packed matrix's tile height and tile count
    AttnArgs at;            // OP_ATTN
    // Input dependency: wait until *wait_cnt >= (epoch + 1) * wait_units (nullptr: none; the
    // tensor-parallel reduce prologue waits on its exchange counter itself).
    const unsigned long long *wait_cnt = nullptr;
    unsigned long long wait_units = 0;
    // Completion: rows (SwiGLU: output pairs) or attention outputs finished are added here.
    unsigned long long *done_cnt = nullptr;
};
struct StepArgs {
    const StepOp *ops = nullptr;  // device array
    int nops = 0;
    int S = 2, NC = 1;            // ring slots, GEMV consumer warps
    // copies a CTA's producers keep in flight (issued, not landed; a multiple of kStepProducers, or 0: as
    // many as the ring has free slots), so that the weight stream does not queue the step's own
    // dependent stores and loads behind it at the memory controllers
    int inflight = 0;
    // the same while the compute warps wait for an op's input, build its activation or run attention
    // (StepCtl::crit; 0: inflight throughout)
    int inflight_crit = 0;
    size_t slot = 0;              // bytes of one ring slot (>= the largest stage)
    size_t xoff = 0;              // activation / attention scratch
    size_t ctl_off = 0;           // control block
    size_t smem = 0;              // dynamic shared memory
    const unsigned long long *epoch = nullptr;  // decode steps completed
    unsigned long long *epoch_rw = nullptr;     // advanced by the classifier's last CTA
    const int *pos = nullptr;
    int seq_len = 0;
    int *err = nullptr;
    unsigned long long *trace = nullptr;  // optional timeline [grid][nops][8] (globaltimer, ns)
    // optional per-stage timeline of ops stage_op0 .. stage_op0 + kStageTraceOps - 1 on the first
    // kStageTraceCtas CTAs: [op][cta][stage][4] = data landed, terms computed, running sums received, passed on
    unsigned long long *stage_trace = nullptr;
    int stage_op0 = 0;
};
constexpr int kStageTraceOps = 5, kStageTraceCtas = 4, kStageTraceStages = 64;
constexpr size_t kStageTraceEntries = (size_t)kStageTraceOps * kStageTraceCtas * kStageTraceStages * 4;
size_t step_ctl_bytes();
size_t step_attn_scratch_bytes(int n_heads, int n_kv_heads, int head_size);
// attention items one wave of the persistent step runs: num_ctas x the CTA's groups of `warps` warps
int step_attn_item_slots(int num_ctas, int warps);
int step_threads();
int step_max_ctas_per_sm(size_t smem);
cudaError_t launch_step(const StepArgs &sa, int grid, cudaStream_t st);
// Prompt prefill of positions pos0 .. pos0+ntok-1 with the decode step's arithmetic (step.cu): the
// Q8_0 activation of every token (a.x: [ntok][n] rows; xq [ntok][n], xs [ntok][n/32] out), the RoPE +
// KV-cache write of every position, and the attention of every position (qkv / out rows `*_stride`
// floats apart; per-position split scratch work_stride floats and count_stride counters apart) with
// the decode step's split plan, batch order and merges, K/V rows loaded once for a group of positions.
cudaError_t launch_prefill_act(const GemvArgs &a, int ntok, const int *tokens, int8_t *xq, float *xs, cudaStream_t st);
cudaError_t launch_prefill_kv(const AttnArgs &a, int pos0, int ntok, size_t qkv_stride, cudaStream_t st);
// Prefill attention items: the prompt positions that share the decode step's attention form and split plan
// (split count and chunk; any chunk when there is one split) go together, at most kPrefillRows (query, head) rows, and
// one item = (group, KV head, split).
constexpr int kPrefillRows = 8;
struct PrefillGroup {
    int first, count;   // positions first .. first+count-1
    int nsplit, chunk;  // their split plan (one split: chunk = the last position + 1)
    int item0;          // index of the group's first item
    int warps;          // the attention form of their positions (kAttnNarrowWarps or kAttnWideWarps)
};
// Tensor-parallel prefill exchange (wo / w2 partial sums of a chunk, over NVLink peer memory):
// scatter: dst[q] + off receives this rank's nf partial floats, for every rank q (system fence after);
// signal:  every rank's counter cnt[q] + 1 (after the scatter, in stream order);
// wait:    until *cnt >= target (bounded; DK_ERR_COMM in *err when a rank never arrives);
// reduce:  x[i] = x[i] + (recv[0][i] + recv[1][i] + ...), ranks in order, recv[q] = recv + q * stride.
cudaError_t launch_prefill_scatter(const float *src, float *const *dst, int world, size_t off, size_t nf, cudaStream_t st);
cudaError_t launch_prefill_signal(unsigned long long *const *cnt, int world, cudaStream_t st);
cudaError_t launch_prefill_wait(const unsigned long long *cnt, unsigned long long target, int *err, cudaStream_t st);
cudaError_t launch_prefill_reduce(float *x, const float *recv, size_t stride, int world, size_t nf, cudaStream_t st);
// Fills groups[0 .. n) (capacity ntok) for positions pos0 .. pos0+ntok-1 with the persistent step's attention
// form and split plan (step_attn_plan); returns n, *items = total items, *narrow_items = the items of the narrow
// groups, which come first.
int prefill_attn_plan(const AttnArgs &a, int pos0, int ntok, PrefillGroup *groups, long long *items,
                      long long *narrow_items = nullptr);
cudaError_t launch_prefill_attn(const AttnArgs &a, int pos0, const PrefillGroup *d_groups, int ngroups,
                                long long items, long long narrow_items, size_t qkv_stride, size_t out_stride,
                                size_t work_stride, size_t count_stride, cudaStream_t st);

}  // namespace dk
