/*
 * diolkos.h -- the C ABI of the B200 decode path (libdiolkos.so).
 *
 * Plain pointers, sizes and int status codes; no C++ or torch types.  "Device" pointers are CUDA
 * device addresses on the current device; `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream).  Every entry point returns DK_OK (0) or a DK_ERR_* code, and
 * dk_last_error() describes the most recent failure of the calling thread.
 *
 * The reference's own C API (transformer.h, safetensors.h, tensor.h, utils.h, sampler.h,
 * tokenizer.h in this directory) is implemented on top of these entry points by the same library.
 */
#ifndef DIOLKOS_H
#define DIOLKOS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The device-side error word uses the same bits. */
#define DK_OK            0
#define DK_ERR_INVALID   0x01 /* bad argument or shape                                  */
#define DK_ERR_CUDA      0x02 /* a CUDA runtime call failed                              */
#define DK_ERR_TIMEOUT   0x04 /* a bounded device-side wait gave up                      */
#define DK_ERR_NOMEM     0x08 /* device or host allocation failed                        */
#define DK_ERR_IO        0x10 /* file could not be read or written                       */
#define DK_ERR_STATE     0x20 /* call not valid in the object's current state             */
#define DK_ERR_COMM      0x40 /* a peer (tensor-parallel rank) did not answer in time     */

const char *dk_last_error(void);
int dk_device_count(void);

/* ---------------------------------------------------------------------------------------------
 * Q8_0 format: groups of 32 int8 values with one fp32 scale (value = q * scale).
 * ------------------------------------------------------------------------------------------- */

/* Weight quantiser: replaces convert_bf16_q8_0 (reference src/tensor.c:312-344).  Device
 * pointers; n % 32 == 0.  Bit-exact with the reference build: scale = amax*(1/127),
 * q = rint(x * (1/scale)). */
int dk_quantize_bf16_q8_0(const uint16_t *x, size_t n, int8_t *q, float *scale, void *stream);
/* The same recipe on IEEE half weights: replaces convert_f16_q8_0 (src/tensor.c:278-310). */
int dk_quantize_f16_q8_0(const uint16_t *x, size_t n, int8_t *q, float *scale, void *stream);
/* Activation quantiser: replaces convert_f32_q8_slice_into_offset (src/tensor.c:199-228). */
int dk_quantize_f32_q8_0(const float *x, size_t n, int8_t *q, float *scale, void *stream);
/* Dequantiser: replaces convert_q8_f32_slice_into_offset (src/tensor.c:245-265). */
int dk_dequantize_q8_0(const int8_t *q, const float *scale, size_t n, float *out, void *stream);
/* The exact int32 dot of every 32-element group of a [d x n] Q8_0 matrix with a Q8_0 vector
 * (the inner loop of matmul_Q8_0, src/utils.c:122-127): dots[i*(n/32)+g]. */
int dk_q8_0_group_dots(const int8_t *xq, const int8_t *wq, int n, int d, int32_t *dots, void *stream);

/* Packed device weight layout used by the GEMV (no reference counterpart: the reference keeps
 * the planar cache layout in host memory).  A [d x n] matrix is cut into 512-column blocks; per
 * row and block a SEGMENT holds the block's int8 values then its fp32 scales, padded to 16 bytes
 * (576 bytes for a full block).  Rows are grouped into tiles of dk_q8_tile_rows(d) rows (chosen so
 * that every SM of the current device streams the same number of rows); a tile stores block 0 of
 * its rows, then block 1, ..., and the 16-byte chunks inside a segment are XOR-swizzled by the
 * row's index in its tile.  The last tile is zero-padded.  The layout depends on the SM count, so
 * pack on the device that runs the GEMV.
 * dk_q8_row_bytes: bytes of all segments of one row (0 for n not a positive multiple of 32). */
size_t dk_q8_row_bytes(int n);
/* Tile height (1..32) of a d-row matrix on the current device. */
int dk_q8_tile_rows(int d);
/* Bytes of the packed [d x n] matrix on the current device (0 for bad shapes). */
size_t dk_q8_packed_bytes(int n, int d);
/* Pack a planar Q8_0 [d x n] matrix (the on-disk cache layout: int8[d*n] then fp32[d*n/32];
 * device pointers, src_q 16-byte aligned) into dst (dk_q8_packed_bytes(n, d) bytes, 16-byte
 * aligned), replacing the reference's load of a Q8_0 tensor from its cache file
 * (src/tensor.c:346-397).  Asynchronous on `stream`. */
int dk_q8_pack(uint8_t *dst, int n, int d, const int8_t *src_q, const float *src_scale, void *stream);

/* matmul_Q8_0 (src/utils.c:106-138) on packed weights: out[d] = W[d x n] * quant(x[n]).
 * Device pointers.  Output bit-exact with the reference build (same group order, same
 * rounding). */
int dk_matmul_q8_0(float *out, const float *x, const uint8_t *w_packed, int n, int d, void *stream);
/* The same GEMV on an activation that is already quantised (xq int8[n], xs fp32[n/32]). */
int dk_matmul_q8_0_q(float *out, const int8_t *xq, const float *xs, const uint8_t *w_packed, int n,
                     int d, void *stream);
/* `count` GEMVs of the same activation x against count packed [d x n] matrices (the reference calls
 * matmul once per matrix, e.g. wq, wk, wv on the same xb, src/transformer.c:83-85): out[i*d .. (i+1)*d)
 * = W_i * quant(x), each bit-identical to dk_matmul_q8_0.  One launch per 32 matrices: every SM runs two
 * CTAs that stream their tiles of alternate matrices, one matrix after another, through their rings (the
 * activation built once); a later launch starts while the previous one runs and waits for it only before
 * its first output store. */
int dk_matmul_q8_0_batch(float *out, const float *x, const uint8_t *const *w_packed, int count, int n,
                         int d, void *stream);
/* matmul_Q8_0 (src/utils.c:106-138) for a batch of `ntok` already-quantised activation vectors
 * (prompt prefill; the reference calls matmul once per token): out[t*d + i] = W[i] . x_t (accumulate != 0: +=), from the
 * same packed matrix as dk_matmul_q8_0.  xq int8[ntok][n] (16-byte aligned), xs fp32[ntok][n/32].
 * The int32 group dots come from the tensor cores (tcgen05.mma kind::i8, one MMA per 32-value group);
 * every output is bit-identical to dk_matmul_q8_0_q on that token. */
int dk_matmul_q8_0_tokens(float *out, const int8_t *xq, const float *xs, const uint8_t *w_packed, int n, int d,
                          int ntok, int accumulate, void *stream);
/* Token sampling (reference sample(), src/sampler.c:108-131) on device logits[n]: temperature 0 is
 * argmax (first index wins ties); otherwise softmax(logits / temperature), then with `coin` in
 * [0, 1) multinomial sampling in index order (topp <= 0 or >= 1) or top-p sampling over the tokens
 * sorted by decreasing probability.  Writes the token to the device int *out and, when probs is not
 * NULL (temperature > 0), the probabilities to device probs[n] -- what the reference leaves in its
 * logits buffer; probs may be the logits buffer itself.  One CTA; no scratch. */
int dk_sample(const float *logits, int n, float temperature, float topp, float coin, float *probs, int *out,
              void *stream);
/* softmax_f32 (src/utils.c:39-57) in place on device x[n]. */
int dk_softmax(float *x, int n, void *stream);
/* rmsnorm (src/utils.c:59-76), device pointers; o may alias x. */
int dk_rmsnorm(float *o, const float *x, const float *w, int n, void *stream);

/* The attention block of one decode step of one layer: replaces src/transformer.c:87-193 of
 * forward (RoPE on q and k, k and v written into the cache at pos, then softmax(q.k/sqrt(hs))
 * weighted sum of v for every query head over positions 0..pos), as split-K flash-decoding.
 * Device pointers:
 *   qkv     fp32 [n_heads*hs + 2*n_kv_heads*hs] = q | k | v, the wq/wk/wv outputs before RoPE;
 *   rope    fp32 [seq_len][hs/2][2] = (cosf(p*f_j), sinf(p*f_j)), f_j = 1/powf(10000, 2j/(float)hs);
 *   k_cache, v_cache  [n_kv_heads][seq_len][hs] of kv_type (DK_KV_BF16 truncating, or DK_KV_F32);
 *   pos     int, the position (0 <= pos < seq_len; read on the device, so a captured call can be
 *           replayed for every position);
 *   out     fp32 [n_heads*hs];
 *   work    scratch of dk_attention_work_bytes(...) bytes, 256-byte aligned, zero-filled before its
 *           first use; every call leaves it ready for the next one.
 * Calls that share `work` must be ordered (one stream). */
size_t dk_attention_work_bytes(int n_heads, int n_kv_heads, int head_size, int seq_len);
int dk_attention_decode(float *out, const float *qkv, const float *rope, void *k_cache, void *v_cache,
                        int kv_type, const int *pos, int n_heads, int n_kv_heads, int head_size,
                        int seq_len, void *work, void *stream);
/* dk_attention_decode without a `work` argument and without allocating anything.  No reference
 * counterpart: the reference's attention needs no scratch.  The scratch lives in a static device
 * array of 4 MiB (4194304 bytes) per device, holding the split partials, the arrival counters and
 * an error word; shapes that need more (dk_attention_work_bytes(...) + 256 bytes) are rejected
 * with DK_ERR_INVALID.  The same arguments give the same bits as dk_attention_decode.
 *   - The first call on each device does setup: it looks up the array's device address (which may
 *     load this module onto the device).  Make that first call before any stream capture.
 *   - Every call clears the counters and the error word with cudaMemsetAsync on `stream`; it calls
 *     no cudaMalloc, cudaFree or other allocating routine.
 *   - All calls on one device share the one array: calls that overlap in time (other streams,
 *     other threads) race on it and give wrong results.  Order them on one stream. */
int dk_attention_decode_noalloc(float *out, const float *qkv, const float *rope, void *k_cache,
                                void *v_cache, int kv_type, const int *pos, int n_heads,
                                int n_kv_heads, int head_size, int seq_len, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Decode engine: one LLaMA-2 model resident on one GPU (or one tensor-parallel shard), whose
 * whole per-token step (reference forward, src/transformer.c:55-239) is one CUDA graph.
 * ------------------------------------------------------------------------------------------- */
typedef struct dk_model dk_model;

/* Weight identifiers (HF tensor names in the comments). */
enum dk_weight {
    DK_W_EMB = 0,   /* model.embed_tokens.weight        Q8_0 [vocab x dim]  */
    DK_W_RMS_FINAL, /* model.norm.weight                F32  [dim]          */
    DK_W_WCLS,      /* lm_head.weight                   Q8_0 [vocab x dim]  */
    DK_W_RMS_ATT,   /* layers.L.input_layernorm         F32  [dim]          */
    DK_W_WQ,        /* layers.L.self_attn.q_proj        Q8_0 [dim x dim]    */
    DK_W_WK,        /* layers.L.self_attn.k_proj        Q8_0 [kv_dim x dim] */
    DK_W_WV,        /* layers.L.self_attn.v_proj        Q8_0 [kv_dim x dim] */
    DK_W_WO,        /* layers.L.self_attn.o_proj        Q8_0 [dim x dim]    */
    DK_W_RMS_FFN,   /* layers.L.post_attention_layernorm F32 [dim]          */
    DK_W_W1,        /* layers.L.mlp.gate_proj           Q8_0 [hidden x dim] */
    DK_W_W2,        /* layers.L.mlp.down_proj           Q8_0 [dim x hidden] */
    DK_W_W3,        /* layers.L.mlp.up_proj             Q8_0 [hidden x dim] */
    DK_W_COUNT
};

/* KV-cache element type. */
#define DK_KV_BF16 0 /* the reference's bf16-truncating cache (src/transformer.c:25-26, :145-146) */
#define DK_KV_F32  1 /* fp32 cache                                                            */

/* cfg = {dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len} (the reference's
 * Config, src/transformer.h:14-22).  Allocates all device memory of the model on `device`.
 * tp_rank / tp_world select this process's tensor-parallel shard (0 / 1 for one GPU; up to 8 ranks,
 * one process per GPU of one node), the split the reference's client/worker topology makes across
 * machines (src/bin/client.c): attention heads and w1/w3 rows per rank, wo and w2 by columns (their
 * partial outputs summed over the ranks), classifier rows per rank, embedding and norms on every
 * rank.  heads, kv heads must divide by tp_world; hidden/tp_world and head_size*heads/tp_world must
 * be multiples of 32. */
dk_model *dk_model_create(const int *cfg, int kv_type, int device, int tp_rank, int tp_world);
/* Tensor parallel only (tp_world > 1), before dk_model_finalize.  Each rank exports the CUDA IPC
 * handle of its exchange area (DK_COMM_HANDLE_BYTES bytes), the ranks share them (any transport),
 * and each rank connects to all of them: handles = tp_world handles in rank order.  The per-layer
 * sums then travel inside the GEMVs over NVLink peer memory: no collective library is involved.
 * All ranks must then run the same decode steps (forward / generate / enqueue_steps) in the same
 * order; a rank that stops makes the others' waits time out with DK_ERR_COMM. */
#define DK_COMM_HANDLE_BYTES 64
int dk_model_comm_handle(dk_model *m, void *handle);
int dk_model_comm_connect(dk_model *m, const void *handles);
void dk_model_destroy(dk_model *m);
/* Set one weight from HOST memory.  Q8_0 weights: q = int8[rows*cols], scale = fp32[rows*cols/32]
 * in the planar cache layout, full (unsharded) matrix; the engine keeps this rank's shard.
 * F32 weights: q = float[n], scale = NULL.  layer = -1 for the non-layer weights. */
int dk_model_set_weight(dk_model *m, int which, int layer, const void *q, const float *scale);
/* Same, with the planar Q8_0 (or F32) data in DEVICE memory of the model's GPU.  Both calls return
 * once the data has been copied: the caller may free or reuse its buffers afterwards.  The copy runs
 * on the model's own (non-blocking) stream, so the work that produced the data must be complete
 * before the call (e.g. synchronise the stream that wrote it). */
int dk_model_set_weight_device(dk_model *m, int which, int layer, const void *q, const float *scale);
/* Check that every weight is present and capture the per-token CUDA graph. */
int dk_model_finalize(dk_model *m);

/* One decode step (reference forward(transformer, token, pos)): writes vocab logits to the HOST
 * buffer `logits` (NULL: skip the copy).  With tensor parallelism each rank writes only its own
 * classifier rows (the slice of logits[vocab_size] it computes). */
int dk_model_forward(dk_model *m, int token, int pos, float *logits);
/* Greedy generation with the reference generate() rules (src/bin/localinfer.c:42-99): prompt
 * tokens are forced, then argmax tokens (first index wins ties) are fed back; stops after `steps`
 * positions or when the sampled token is 1.  The whole loop runs on the GPU: the forced positions
 * (all prompt tokens but the last) run as one batched prefill on the tensor cores, whose KV-cache
 * entries equal the decode step's bit for bit (tensor parallel too: call it on every rank);
 * DIOLKOS_PREFILL=0 steps them instead.  out receives the generated (non-forced) tokens, *n_out
 * their count.  Host buffers. */
int dk_model_generate(dk_model *m, const int *prompt, int n_prompt, int steps, int *out, int *n_out);

/* Lower-level control used by benchmarks: enqueue decode steps for positions
 * [pos0, pos0 + n_steps) with tokens taken from the device token buffer (set by dk_model_set_tokens)
 * and argmax results written back into it; nothing is synchronised. */
int dk_model_set_tokens(dk_model *m, const int *tokens, int n_tokens, int n_forced);
int dk_model_enqueue_steps(dk_model *m, int pos0, int n_steps);
/* Prompt prefill: runs positions [pos0, pos0 + n_positions) through every layer at once for the
 * tokens in the device token buffer, writing their KV-cache entries exactly as decode steps at those
 * positions would (the reference forwards prompt tokens one by one, src/bin/localinfer.c:60-73);
 * no logits.  Int8 tensor-core matmuls (tcgen05), chunks of up to 256 positions.  Tensor parallel:
 * every rank makes the same call; the wo / w2 partial sums cross NVLink once per layer each and are
 * summed in rank order like the decode step's (a rank that never arrives makes the others' waits end
 * with DK_ERR_COMM).  Needs the persistent decode step (DK_ERR_STATE otherwise).  After an exchange
 * of a tensor-parallel prefill failed to enqueue, the ranks' exchange counts may disagree, so that
 * model refuses further prefills (DK_ERR_STATE) and dk_model_generate steps its prompt instead.
 * Enqueued, not synchronised. */
int dk_model_prefill(dk_model *m, int pos0, int n_positions);
int dk_model_get_tokens(dk_model *m, int *tokens, int n_tokens);
int dk_model_sync(dk_model *m);
/* The CUDA stream the engine launches on (cudaStream_t as void*). */
void *dk_model_stream(dk_model *m);
/* Device error word (DK_ERR_* bits raised by kernels); reading it synchronises the stream. */
int dk_model_device_error(dk_model *m);
/* Number of kernels one decode step launches (for launch accounting). */
int dk_model_kernels_per_step(dk_model *m);
/* Diagnostics for per-layer parity checks (persistent step only).  dk_model_dump_enable(m, 1) makes
 * every later decode step record, for each GEMV of the step in order -- per layer q|k|v, wo, w1|w3,
 * w2, then the classifier -- its fp32 input vector (the residual stream for the rmsnorm prologues, the
 * attention output for wo, the SwiGLU output for w2; n floats) and the Q8_0 activation it multiplied
 * (n int8 values, n/32 fp32 scales): the checkpoints of the reference's forward() at its rmsnorm and
 * matmul calls (src/transformer.c:76-237).  dk_model_dump_read copies the last step's record into
 * host buffers holding the ops' n summed (in, q) and that sum / 32 (s); NULL skips one.  Costs one
 * branch per op when off; (0) turns it off again. */
int dk_model_dump_enable(dk_model *m, int on);
int dk_model_dump_read(dk_model *m, float *in, int8_t *q, float *s);
/* Diagnostics: overwrite the KV-cache rows of positions [pos0, pos0 + n_pos) of one layer with host
 * rows in the reference's cache layout (src/transformer.c:25-26, :145-146: [n_pos][kv_dim], all KV
 * heads; a tensor-parallel rank takes its own heads) of src_type DK_KV_BF16 (bf16 bits) or DK_KV_F32,
 * converted to the cache's type as the decode step stores it (bf16 truncates, bf16 -> fp32 is exact).
 * Lets a test give the engine an oracle's own history before a step.  Synchronous. */
int dk_model_kv_write(dk_model *m, int layer, int pos0, int n_pos, const void *k, const void *v, int src_type);
/* Diagnostics: this rank's KV-cache rows of positions [pos0, pos0 + n_pos) of one layer, in the
 * reference's layout ([n_pos][this rank's KV heads * hs]) and the cache's element type.  Synchronous. */
int dk_model_kv_read(dk_model *m, int layer, int pos0, int n_pos, void *k, void *v);
/* Diagnostics: the persistent step's timeline of the last decode step, when the model was created
 * with DIOLKOS_STEP_TRACE=1 in the environment: out[(cta * n_ops + op) * 8 + k] = GPU global timer (ns)
 * when, on that CTA, k = 0: the op's input was ready, 1: its activation was built, 2: it finished,
 * 3: the op's last weight stage was issued, 4: the input counter was seen (0: not recorded).
 * *grid and *n_ops give the dimensions.  When n also covers 5 * 4 * 64 * 4 more entries, these follow:
 * the GEMV consumers' per-stage timeline of the second layer's five ops on CTAs 0..3,
 * [op][cta][stage][k] with k = 0: the stage's weights landed, 1: its group terms were computed, 2: the
 * running row sums of the previous stage were received, 3: this stage's sums were passed on. */
int dk_model_trace(dk_model *m, unsigned long long *out, size_t n, int *grid, int *n_ops);
/* Diagnostics: the timeline of the last pipelined tensor-core matmul launched on this device while
 * DIOLKOS_GEMM_TRACE=1 was set at the first launch: out[(cta * blocks + b) * 5 + k] = GPU global timer
 * (ns) when, for 512-column block b of that CTA, k = 0: its copies were issued, 1: the MMA thread saw
 * them land, 2: its last MMA was issued, 3: fold warp 2 saw them land, 4: fold warp 2 finished it
 * (0: not recorded).  *ctas and *blocks give the dimensions (the first 148 CTAs, 32 blocks). */
int dk_gemm_trace(unsigned long long *out, size_t n, int *ctas, int *blocks);
/* Diagnostics (host only, no GPU): the attention's split plan over T positions (the count of splits and
 * their length; the decode step's attention, src/transformer.c:149-193, split for the GPU).
 * dk_attn_split_plan: one plan (the standalone attention kernel's form).
 * dk_step_attn_plan: the persistent step's two forms, plan[5] = {narrow max splits, narrow shortest
 * split, wide max splits, wide shortest split, wide_from}: T <= wide_from takes the narrow form (items of
 * 2 warps), beyond the wide one (items of 10 warps, the chunk rounded up to whole 8-position batches);
 * returns the item's warps.
 * dk_prefill_attn_plan: the prefill attention's position groups for positions pos0 .. pos0+ntok-1 under
 * the step's plan: groups_out receives 6 ints per group (first position, count, split count, chunk,
 * first item index, item warps), capacity ntok groups; returns the group count, *items the total
 * (group, KV head, split) items and *narrow_items those of the narrow groups, which come first. */
int dk_attn_split_plan(int T, int max_splits, int min_chunk, int *nsplit, int *chunk);
int dk_step_attn_plan(int T, const int *plan, int *nsplit, int *chunk);
int dk_prefill_attn_plan(int n_heads, int n_kv_heads, const int *plan, int pos0, int ntok, int *groups_out,
                         long long *items, long long *narrow_items);
/* Bytes of weights one decode step reads on this rank. */
size_t dk_model_weight_bytes(dk_model *m);

#ifdef __cplusplus
}
#endif
#endif /* DIOLKOS_H */
