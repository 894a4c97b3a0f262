"""Kernel-level operators of the C ABI on torch CUDA tensors (torch is only the memory plumbing).

Each function mirrors one reference function (cited) and calls the CUDA kernel through
libdiolkos.so; there is no fallback.
"""
from __future__ import annotations

import torch

from ._native import check, lib, stream_ptr


def _ptr(t: torch.Tensor) -> int:
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return t.data_ptr()


def quantize_bf16(x_bits: torch.Tensor):
    """convert_bf16_q8_0 (src/tensor.c:312-344) on bf16 bit patterns (int16/uint16/bfloat16)."""
    n = x_bits.numel()
    q = torch.empty(n, dtype=torch.int8, device=x_bits.device)
    s = torch.empty(n // 32, dtype=torch.float32, device=x_bits.device)
    check(lib().dk_quantize_bf16_q8_0(_ptr(x_bits), n, _ptr(q), _ptr(s), stream_ptr()))
    return q, s


def quantize_f32(x: torch.Tensor):
    """convert_f32_q8_slice_into_offset (src/tensor.c:199-228)."""
    n = x.numel()
    q = torch.empty(n, dtype=torch.int8, device=x.device)
    s = torch.empty(n // 32, dtype=torch.float32, device=x.device)
    check(lib().dk_quantize_f32_q8_0(_ptr(x), n, _ptr(q), _ptr(s), stream_ptr()))
    return q, s


def dequantize(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """convert_q8_f32_slice_into_offset (src/tensor.c:245-265)."""
    out = torch.empty(q.numel(), dtype=torch.float32, device=q.device)
    check(lib().dk_dequantize_q8_0(_ptr(q), _ptr(s), q.numel(), _ptr(out), stream_ptr()))
    return out


def group_dots(xq: torch.Tensor, wq: torch.Tensor, n: int, d: int) -> torch.Tensor:
    """The exact int32 group dots of matmul_Q8_0 (src/utils.c:122-127), shape [d, n/32]."""
    dots = torch.empty((d, n // 32), dtype=torch.int32, device=xq.device)
    check(lib().dk_q8_0_group_dots(_ptr(xq), _ptr(wq), n, d, _ptr(dots), stream_ptr()))
    return dots


def row_bytes(n: int) -> int:
    return int(lib().dk_q8_row_bytes(n))


def tile_rows(d: int) -> int:
    """Tile height of a packed d-row matrix on the current device."""
    return int(lib().dk_q8_tile_rows(d))


def packed_bytes(n: int, d: int) -> int:
    return int(lib().dk_q8_packed_bytes(n, d))


def pack(q: torch.Tensor, s: torch.Tensor, n: int, d: int) -> torch.Tensor:
    """Planar Q8_0 [d x n] (cache layout) -> the GEMV's packed tile layout."""
    w = torch.empty(packed_bytes(n, d), dtype=torch.uint8, device=q.device)
    check(lib().dk_q8_pack(_ptr(w), n, d, _ptr(q), _ptr(s), stream_ptr()))
    return w


def matmul(x: torch.Tensor, w_packed: torch.Tensor, n: int, d: int, out: torch.Tensor | None = None):
    """matmul_Q8_0 (src/utils.c:106-138): quantise x, then GEMV against packed weights."""
    if out is None:
        out = torch.empty(d, dtype=torch.float32, device=x.device)
    check(lib().dk_matmul_q8_0(_ptr(out), _ptr(x), _ptr(w_packed), n, d, stream_ptr()))
    return out


def matmul_q(xq: torch.Tensor, xs: torch.Tensor, w_packed: torch.Tensor, n: int, d: int,
             out: torch.Tensor | None = None):
    """The GEMV on an already-quantised activation."""
    if out is None:
        out = torch.empty(d, dtype=torch.float32, device=xq.device)
    check(lib().dk_matmul_q8_0_q(_ptr(out), _ptr(xq), _ptr(xs), _ptr(w_packed), n, d, stream_ptr()))
    return out


def matmul_tokens(xq: torch.Tensor, xs: torch.Tensor, w_packed: torch.Tensor, n: int, d: int,
                  out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """dk_matmul_q8_0_tokens: the tensor-core matmul of ntok quantised activation rows (xq int8
    [ntok, n], xs fp32 [ntok, n/32]) against a packed matrix; returns fp32 [ntok, d]."""
    ntok = xq.shape[0]
    if out is None:
        out = torch.empty((ntok, d), dtype=torch.float32, device=xq.device)
    check(lib().dk_matmul_q8_0_tokens(out.data_ptr(), xq.data_ptr(), xs.data_ptr(), w_packed.data_ptr(), n, d, ntok,
                                      1 if accumulate else 0, stream_ptr()))
    return out


def matmul_batch(x: torch.Tensor, ws: list, n: int, d: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """GEMVs of one activation against several packed matrices, back to back: out[i] = W_i * quant(x)."""
    import ctypes

    if out is None:
        out = torch.empty((len(ws), d), dtype=torch.float32, device=x.device)
    ptrs = (ctypes.c_void_p * len(ws))(*[_ptr(w) for w in ws])
    check(lib().dk_matmul_q8_0_batch(_ptr(out), _ptr(x), ptrs, len(ws), n, d, stream_ptr()))
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """rmsnorm (src/utils.c:59-76)."""
    o = torch.empty_like(x)
    check(lib().dk_rmsnorm(_ptr(o), _ptr(x), _ptr(w), x.numel(), stream_ptr()))
    return o


def attention_work_bytes(n_heads: int, n_kv_heads: int, head_size: int, seq_len: int) -> int:
    return int(lib().dk_attention_work_bytes(n_heads, n_kv_heads, head_size, seq_len))


def attention_decode(qkv: torch.Tensor, rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     pos: torch.Tensor, n_heads: int, n_kv_heads: int, head_size: int, seq_len: int,
                     work: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The attention block of forward (src/transformer.c:87-193) for one position: RoPE, KV-cache write
    at pos (an int32 device tensor), softmax attention over 0..pos.  The cache type follows the cache
    tensors' dtype (float32, or bfloat16/int16 bit patterns)."""
    kv_type = 1 if k_cache.dtype == torch.float32 else 0
    if out is None:
        out = torch.empty(n_heads * head_size, dtype=torch.float32, device=qkv.device)
    check(lib().dk_attention_decode(_ptr(out), _ptr(qkv), _ptr(rope), _ptr(k_cache), _ptr(v_cache), kv_type,
                                    _ptr(pos), n_heads, n_kv_heads, head_size, seq_len, _ptr(work), stream_ptr()))
    return out


def attention_decode_noalloc(qkv: torch.Tensor, rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                             pos: torch.Tensor, n_heads: int, n_kv_heads: int, head_size: int, seq_len: int,
                             out: torch.Tensor) -> torch.Tensor:
    """attention_decode with the library's static device scratch (no allocation anywhere: `out` is
    the caller's)."""
    kv_type = 1 if k_cache.dtype == torch.float32 else 0
    check(lib().dk_attention_decode_noalloc(_ptr(out), _ptr(qkv), _ptr(rope), _ptr(k_cache), _ptr(v_cache), kv_type,
                                            _ptr(pos), n_heads, n_kv_heads, head_size, seq_len, stream_ptr()))
    return out
