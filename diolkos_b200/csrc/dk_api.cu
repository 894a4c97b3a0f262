// dk_api.cu -- kernel-level entry points of the C ABI (include/diolkos.h) and error reporting.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "dk_internal.h"

#include <vector>

namespace dk {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return DK_OK;
    return set_error(DK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int current_num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace dk

using namespace dk;

extern "C" {

const char *dk_last_error(void) { return g_err; }

int dk_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

static int check_aligned(const void *p, size_t a, const char *name) {
    if (reinterpret_cast<uintptr_t>(p) % a)
        return set_error(DK_ERR_INVALID, "%s must be %zu-byte aligned", name, a);
    return DK_OK;
}

int dk_quantize_bf16_q8_0(const uint16_t *x, size_t n, int8_t *q, float *scale, void *stream) {
    if (n % 32) return set_error(DK_ERR_INVALID, "dk_quantize_bf16_q8_0: n=%zu is not a multiple of 32", n);
    if (!x || !q || !scale) return set_error(DK_ERR_INVALID, "dk_quantize_bf16_q8_0: null pointer");
    if (int r = check_aligned(x, 16, "x")) return r;
    if (int r = check_aligned(q, 16, "q")) return r;
    return cuda_status(launch_quant_bf16(x, n, q, scale, (cudaStream_t)stream), "dk_quantize_bf16_q8_0");
}

int dk_quantize_f16_q8_0(const uint16_t *x, size_t n, int8_t *q, float *scale, void *stream) {
    if (n % 32) return set_error(DK_ERR_INVALID, "dk_quantize_f16_q8_0: n=%zu is not a multiple of 32", n);
    if (!x || !q || !scale) return set_error(DK_ERR_INVALID, "dk_quantize_f16_q8_0: null pointer");
    if (int r = check_aligned(x, 16, "x")) return r;
    if (int r = check_aligned(q, 16, "q")) return r;
    return cuda_status(launch_quant_f16(x, n, q, scale, (cudaStream_t)stream), "dk_quantize_f16_q8_0");
}

int dk_quantize_f32_q8_0(const float *x, size_t n, int8_t *q, float *scale, void *stream) {
    if (n % 32) return set_error(DK_ERR_INVALID, "dk_quantize_f32_q8_0: n=%zu is not a multiple of 32", n);
    if (!x || !q || !scale) return set_error(DK_ERR_INVALID, "dk_quantize_f32_q8_0: null pointer");
    if (int r = check_aligned(x, 16, "x")) return r;
    if (int r = check_aligned(q, 16, "q")) return r;
    return cuda_status(launch_quant_f32(x, n, q, scale, (cudaStream_t)stream), "dk_quantize_f32_q8_0");
}

int dk_dequantize_q8_0(const int8_t *q, const float *scale, size_t n, float *out, void *stream) {
    if (n % 32) return set_error(DK_ERR_INVALID, "dk_dequantize_q8_0: n=%zu is not a multiple of 32", n);
    if (!q || !scale || !out) return set_error(DK_ERR_INVALID, "dk_dequantize_q8_0: null pointer");
    return cuda_status(launch_dequant(q, scale, n, out, (cudaStream_t)stream), "dk_dequantize_q8_0");
}

int dk_q8_0_group_dots(const int8_t *xq, const int8_t *wq, int n, int d, int32_t *dots, void *stream) {
    if (n <= 0 || n % 32 || d <= 0) return set_error(DK_ERR_INVALID, "dk_q8_0_group_dots: bad shape n=%d d=%d", n, d);
    if (int r = check_aligned(xq, 16, "xq")) return r;
    if (int r = check_aligned(wq, 16, "wq")) return r;
    return cuda_status(launch_group_dots(xq, wq, n, d, dots, (cudaStream_t)stream), "dk_q8_0_group_dots");
}

size_t dk_q8_row_bytes(int n) { return (n > 0 && n % 32 == 0) ? q8_row_bytes(n) : 0; }

int dk_q8_tile_rows(int d) { return d > 0 ? gemv_tile_rows(d, EPI_STORE, current_num_sms()) : 0; }

size_t dk_q8_packed_bytes(int n, int d) {
    if (n <= 0 || n % 32 || d <= 0) return 0;
    return q8_packed_bytes(n, d, gemv_tile_rows(d, EPI_STORE, current_num_sms()));
}

int dk_q8_pack(uint8_t *dst, int n, int d, const int8_t *src_q, const float *src_scale, void *stream) {
    if (n <= 0 || n % 32 || d <= 0) return set_error(DK_ERR_INVALID, "dk_q8_pack: bad shape n=%d d=%d", n, d);
    if (!dst || !src_q || !src_scale) return set_error(DK_ERR_INVALID, "dk_q8_pack: null pointer");
    if (int r = check_aligned(dst, 16, "dst")) return r;
    if (int r = check_aligned(src_q, 16, "src_q")) return r;
    if (int r = check_aligned(src_scale, 4, "src_scale")) return r;
    const int T = gemv_tile_rows(d, EPI_STORE, current_num_sms());
    cudaStream_t st = (cudaStream_t)stream;
    if (int r = cuda_status(cudaMemsetAsync(dst, 0, q8_packed_bytes(n, d, T), st), "dk_q8_pack: memset")) return r;
    return cuda_status(launch_pack_rows(dst, n, T, src_q, src_scale, d, 0, 1, st), "dk_q8_pack");
}

static int matmul_common(float *out, const float *x, const int8_t *xq, const float *xs, const uint8_t *w, int n,
                         int d, void *stream) {
    if (n <= 0 || n % 32 || d <= 0) return set_error(DK_ERR_INVALID, "matmul: bad shape n=%d d=%d", n, d);
    if (!out || !w) return set_error(DK_ERR_INVALID, "matmul: null pointer");
    if (int r = check_aligned(w, 16, "w_packed")) return r;
    GemvArgs a;
    a.w = w;
    a.n = n;
    a.d = d;
    a.out = out;
    a.err = device_error_word();
    if (!a.err) return set_error(DK_ERR_CUDA, "matmul: could not allocate the device error word");
    if (x) {
        a.pro = PRO_F32;
        a.x = x;
    } else {
        if (int r = check_aligned(xq, 16, "xq")) return r;
        a.pro = PRO_Q8;
        a.xq = xq;
        a.xs = xs;
    }
    a.epi = EPI_STORE;
    if (!gemv_supported(n, d, EPI_STORE))
        return set_error(DK_ERR_INVALID, "matmul: unsupported shape n=%d d=%d (n must be a multiple of 32 and fit the shared-memory budget)", n, d);
    const GemvPlan p = plan_gemv(n, d, EPI_STORE, current_num_sms());
    return cuda_status(launch_gemv(a, p, (cudaStream_t)stream, false), "matmul");
}

int dk_matmul_q8_0(float *out, const float *x, const uint8_t *w_packed, int n, int d, void *stream) {
    if (!x) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0: null x");
    return matmul_common(out, x, nullptr, nullptr, w_packed, n, d, stream);
}

int dk_matmul_q8_0_q(float *out, const int8_t *xq, const float *xs, const uint8_t *w_packed, int n, int d,
                     void *stream) {
    if (!xq || !xs) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_q: null activation");
    return matmul_common(out, nullptr, xq, xs, w_packed, n, d, stream);
}

size_t dk_attention_work_bytes(int n_heads, int n_kv_heads, int head_size, int seq_len) {
    if (!attn_supported(n_heads, n_kv_heads, head_size) || seq_len <= 0) return 0;
    return attn_work_bytes(n_heads, n_kv_heads, head_size, attn_max_splits(seq_len, n_kv_heads, current_num_sms()));
}

int dk_attention_decode(float *out, const float *qkv, const float *rope, void *k_cache, void *v_cache, int kv_type,
                        const int *pos, int n_heads, int n_kv_heads, int head_size, int seq_len, void *work,
                        void *stream) {
    if (!attn_supported(n_heads, n_kv_heads, head_size) || seq_len <= 0)
        return set_error(DK_ERR_INVALID, "dk_attention_decode: unsupported shape heads=%d kv_heads=%d head_size=%d",
                         n_heads, n_kv_heads, head_size);
    if (kv_type != DK_KV_BF16 && kv_type != DK_KV_F32)
        return set_error(DK_ERR_INVALID, "dk_attention_decode: bad kv_type %d", kv_type);
    if (!out || !qkv || !rope || !k_cache || !v_cache || !pos || !work)
        return set_error(DK_ERR_INVALID, "dk_attention_decode: null pointer");
    if (reinterpret_cast<uintptr_t>(qkv) % 16 || reinterpret_cast<uintptr_t>(k_cache) % 16 ||
        reinterpret_cast<uintptr_t>(v_cache) % 16)
        return set_error(DK_ERR_INVALID, "dk_attention_decode: qkv, k_cache and v_cache must be 16-byte aligned");
    if (int r = check_aligned(work, 256, "work")) return r;
    AttnArgs a;
    a.qkv = qkv; a.rope = rope; a.k_cache = k_cache; a.v_cache = v_cache; a.out = out; a.pos = pos;
    a.n_heads = n_heads; a.n_kv_heads = n_kv_heads; a.head_size = head_size; a.seq_len = seq_len;
    a.kv_f32 = kv_type == DK_KV_F32;
    a.max_splits = attn_max_splits(seq_len, n_kv_heads, current_num_sms());
    a.min_chunk = kAttnMinChunk;
    a.work = static_cast<float *>(work);
    a.count = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(work) +
                                           attn_count_offset(n_heads, head_size, a.max_splits));
    a.err = device_error_word();
    if (!a.err) return set_error(DK_ERR_CUDA, "dk_attention_decode: could not allocate the device error word");
    return cuda_status(launch_attention(a, (cudaStream_t)stream, false), "dk_attention_decode");
}

int dk_attn_split_plan(int T, int max_splits, int min_chunk, int *nsplit, int *chunk) {
    if (T < 1 || max_splits < 1 || min_chunk < 1 || !nsplit || !chunk)
        return set_error(DK_ERR_INVALID, "dk_attn_split_plan: bad arguments");
    attn_split_plan(T, max_splits, min_chunk, *nsplit, *chunk);
    return DK_OK;
}

static bool step_plan_args(const int *plan, AttnArgs &a) {
    if (!plan || plan[0] < 1 || plan[1] < 1 || plan[2] < 1 || plan[3] < 1 || plan[4] < 0) return false;
    a.narrow_max_splits = plan[0];
    a.narrow_min_chunk = plan[1];
    a.wide_max_splits = plan[2];
    a.wide_min_chunk = plan[3];
    a.wide_from = plan[4];
    a.max_splits = std::max(plan[0], plan[2]);
    return true;
}

int dk_step_attn_plan(int T, const int *plan, int *nsplit, int *chunk) {
    AttnArgs a;
    if (T < 1 || !nsplit || !chunk || !step_plan_args(plan, a))
        return -set_error(DK_ERR_INVALID, "dk_step_attn_plan: bad arguments");
    return step_attn_plan(a, T, *nsplit, *chunk);
}

int dk_prefill_attn_plan(int n_heads, int n_kv_heads, const int *plan, int pos0, int ntok, int *groups_out,
                         long long *items, long long *narrow_items) {
    AttnArgs a;
    if (n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads || pos0 < 0 || ntok < 1 || !groups_out ||
        !step_plan_args(plan, a))
        return -set_error(DK_ERR_INVALID, "dk_prefill_attn_plan: bad arguments");
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    std::vector<PrefillGroup> g((size_t)ntok);
    const int n = prefill_attn_plan(a, pos0, ntok, g.data(), items, narrow_items);
    for (int i = 0; i < n; ++i) {
        int *o = groups_out + 6 * (size_t)i;
        o[0] = g[i].first;
        o[1] = g[i].count;
        o[2] = g[i].nsplit;
        o[3] = g[i].chunk;
        o[4] = g[i].item0;
        o[5] = g[i].warps;
    }
    return n;
}

int dk_gemm_trace(unsigned long long *out, size_t n, int *ctas, int *blocks) {
    int c = 0, b = 0;
    const unsigned long long *buf = gemm_trace_buffer(&c, &b);
    if (ctas) *ctas = c;
    if (blocks) *blocks = b;
    if (!buf) return set_error(DK_ERR_STATE, "dk_gemm_trace: tracing is off (DIOLKOS_GEMM_TRACE=1 before the first launch)");
    const size_t total = (size_t)c * b * kGemmTraceSlots;
    if (!out || n < total) return set_error(DK_ERR_INVALID, "dk_gemm_trace: need %zu entries", total);
    return cuda_status(cudaMemcpy(out, buf, total * 8, cudaMemcpyDeviceToHost), "dk_gemm_trace");
}

int dk_matmul_q8_0_tokens(float *out, const int8_t *xq, const float *xs, const uint8_t *w_packed, int n, int d,
                          int ntok, int accumulate, void *stream) {
    if (!out || !xq || !xs || !w_packed) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_tokens: null pointer");
    if (!gemm_supported(n, d, ntok, EPI_STORE))
        return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_tokens: unsupported shape n=%d d=%d tokens=%d", n, d, ntok);
    if (int r = check_aligned(w_packed, 16, "w_packed")) return r;
    if (int r = check_aligned(xq, 16, "xq")) return r;
    GemmArgs g;
    g.w = w_packed;
    g.n = n;
    g.d = d;
    g.T = q8_tile_rows(d, current_num_sms(), 1);  // the tile height dk_q8_pack used
    g.xq = xq;
    g.xs = xs;
    g.ntok = ntok;
    g.epi = accumulate ? EPI_ADD : EPI_STORE;
    g.out = out;
    g.err = device_error_word();
    if (!g.err) return set_error(DK_ERR_CUDA, "dk_matmul_q8_0_tokens: could not allocate the device error word");
    return cuda_status(launch_gemm(g, (cudaStream_t)stream), "dk_matmul_q8_0_tokens");
}

int dk_matmul_q8_0_batch(float *out, const float *x, const uint8_t *const *w_packed, int count, int n, int d,
                         void *stream) {
    if (count < 0 || (count && !w_packed)) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_batch: bad count or list");
    if (!x || !out) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_batch: null pointer");
    if (n <= 0 || n % 32 || d <= 0 || !gemv_supported(n, d, EPI_STORE))
        return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_batch: unsupported shape n=%d d=%d", n, d);
    for (int i = 0; i < count; ++i) {
        if (!w_packed[i]) return set_error(DK_ERR_INVALID, "dk_matmul_q8_0_batch: null matrix %d", i);
        if (int r = check_aligned(w_packed[i], 16, "w_packed[i]")) return r;
    }
    GemvArgs a;
    a.n = n;
    a.d = d;
    a.pro = PRO_F32;
    a.epi = EPI_STORE;
    a.x = x;
    a.err = device_error_word();
    if (!a.err) return set_error(DK_ERR_CUDA, "dk_matmul_q8_0_batch: could not allocate the device error word");
    // One launch per kGemvBatchMax matrices: each CTA streams its tiles of every matrix of the launch
    // through one ring, the activation built once.  A later launch starts while the previous one runs
    // (x was complete before the first began): it waits for it only before its first output store.
    const GemvPlan p = plan_gemv_batch(n, d, std::min(count, kGemvBatchMax), current_num_sms());
    for (int i0 = 0, k = 0; i0 < count; i0 += kGemvBatchMax, ++k) {
        GemvBatch b;
        b.count = std::min(kGemvBatchMax, count - i0);
        b.groups = b.count > 1 ? 2 : 1;  // two CTAs per SM, alternate matrices: two rings, two row-sum chains
        for (int j = 0; j < b.count; ++j) b.w[j] = w_packed[i0 + j];
        a.out = out + (size_t)i0 * d;
        a.early_input = k > 0;
        if (int r = cuda_status(launch_gemv_batch(a, b, p, (cudaStream_t)stream, k > 0), "dk_matmul_q8_0_batch")) return r;
    }
    return DK_OK;
}

int dk_rmsnorm(float *o, const float *x, const float *w, int n, void *stream) {
    if (n <= 0 || !o || !x || !w) return set_error(DK_ERR_INVALID, "dk_rmsnorm: bad arguments");
    return cuda_status(launch_rmsnorm(o, x, w, n, (cudaStream_t)stream), "dk_rmsnorm");
}

}  // extern "C"
