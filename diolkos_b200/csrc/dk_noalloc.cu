// dk_noalloc.cu -- dk_attention_decode_noalloc: the attention entry point with its scratch in a
// static device array instead of caller- or library-allocated memory.
//
// The array is a file-scope __device__ variable, so it exists once per device, is created when the
// CUDA runtime loads this module on that device, and is never allocated or freed by this code.  Its
// address is looked up with cudaGetSymbolAddress once per device (with that device current) and
// cached.  Per call, the arrival counters and the error word are cleared with cudaMemsetAsync on the
// caller's stream before the kernel is launched; the split partials need no clearing (every split
// writes its own partial before the last split of its KV head reads it).
//
// All calls on one device share the array: calls that overlap in time race on it.
#include <mutex>

#include "dk_internal.h"

namespace dk {
namespace {

constexpr size_t kNoallocScratchBytes = (size_t)4 << 20;  // 4 MiB: partials + counters + error word
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_attn_scratch[kNoallocScratchBytes];

std::mutex g_mu;
void *g_addr[kMaxDevices] = {nullptr};

// Device address of this device's g_attn_scratch (looked up once per device).
int scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(DK_ERR_CUDA, "dk_attention_decode_noalloc: no usable current device");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess)
            return set_error(DK_ERR_CUDA, "dk_attention_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                             dev, cudaGetErrorString(e));
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return DK_OK;
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_attention_decode_noalloc(float *out, const float *qkv, const float *rope, void *k_cache,
                                           void *v_cache, int kv_type, const int *pos, int n_heads, int n_kv_heads,
                                           int head_size, int seq_len, void *stream) {
    if (!attn_supported(n_heads, n_kv_heads, head_size) || seq_len <= 0)
        return set_error(DK_ERR_INVALID,
                         "dk_attention_decode_noalloc: unsupported shape heads=%d kv_heads=%d head_size=%d", n_heads,
                         n_kv_heads, head_size);
    if (kv_type != DK_KV_BF16 && kv_type != DK_KV_F32)
        return set_error(DK_ERR_INVALID, "dk_attention_decode_noalloc: bad kv_type %d", kv_type);
    if (!out || !qkv || !rope || !k_cache || !v_cache || !pos)
        return set_error(DK_ERR_INVALID, "dk_attention_decode_noalloc: null pointer");
    if (reinterpret_cast<uintptr_t>(qkv) % 16 || reinterpret_cast<uintptr_t>(k_cache) % 16 ||
        reinterpret_cast<uintptr_t>(v_cache) % 16)
        return set_error(DK_ERR_INVALID, "dk_attention_decode_noalloc: qkv, k_cache and v_cache must be 16-byte aligned");
    const int max_splits = attn_max_splits(seq_len, n_kv_heads, current_num_sms());
    const size_t work = attn_work_bytes(n_heads, n_kv_heads, head_size, max_splits);
    const size_t need = work + 256;  // + the error word
    if (need > kNoallocScratchBytes)
        return set_error(DK_ERR_INVALID,
                         "dk_attention_decode_noalloc: this shape needs %zu bytes of scratch, more than the %zu-byte "
                         "static scratch; use dk_attention_decode with a caller-provided buffer",
                         need, kNoallocScratchBytes);
    void *base = nullptr;
    if (int r = scratch_address(&base)) return r;
    uint8_t *b = static_cast<uint8_t *>(base);
    const size_t cnt_off = attn_count_offset(n_heads, head_size, max_splits);
    cudaStream_t st = (cudaStream_t)stream;
    // Counters and the error word must start at zero; they sit back to back from cnt_off to need.
    if (int r = cuda_status(cudaMemsetAsync(b + cnt_off, 0, need - cnt_off, st), "dk_attention_decode_noalloc: clear"))
        return r;
    AttnArgs a;
    a.qkv = qkv; a.rope = rope; a.k_cache = k_cache; a.v_cache = v_cache; a.out = out; a.pos = pos;
    a.n_heads = n_heads; a.n_kv_heads = n_kv_heads; a.head_size = head_size; a.seq_len = seq_len;
    a.kv_f32 = kv_type == DK_KV_F32;
    a.max_splits = max_splits;
    a.min_chunk = kAttnMinChunk;
    a.work = reinterpret_cast<float *>(b);
    a.count = reinterpret_cast<unsigned *>(b + cnt_off);
    a.err = reinterpret_cast<int *>(b + work);
    return cuda_status(launch_attention(a, st, false), "dk_attention_decode_noalloc");
}
