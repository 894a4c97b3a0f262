"""ctypes binding of libdiolkos.so (the C ABI in include/diolkos.h).

The library is the product: there is no Python or CPU fallback.  Importing this module on a
machine where the library was not built raises at once.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libdiolkos.so")

DK_OK = 0
DK_ERR_INVALID, DK_ERR_CUDA, DK_ERR_TIMEOUT, DK_ERR_NOMEM, DK_ERR_IO, DK_ERR_STATE, DK_ERR_COMM = (
    0x01, 0x02, 0x04, 0x08, 0x10, 0x20, 0x40)
DK_KV_BF16, DK_KV_F32 = 0, 1
DK_COMM_HANDLE_BYTES = 64
(DK_W_EMB, DK_W_RMS_FINAL, DK_W_WCLS, DK_W_RMS_ATT, DK_W_WQ, DK_W_WK, DK_W_WV, DK_W_WO, DK_W_RMS_FFN,
 DK_W_W1, DK_W_W2, DK_W_W3) = range(12)

# Every symbol include/diolkos.h declares, with (restype, argtypes).
_vp, _sz, _i = C.c_void_p, C.c_size_t, C.c_int
SIGNATURES = {
    "dk_last_error": (C.c_char_p, []),
    "dk_device_count": (_i, []),
    "dk_quantize_bf16_q8_0": (_i, [_vp, _sz, _vp, _vp, _vp]),
    "dk_quantize_f16_q8_0": (_i, [_vp, _sz, _vp, _vp, _vp]),
    "dk_quantize_f32_q8_0": (_i, [_vp, _sz, _vp, _vp, _vp]),
    "dk_dequantize_q8_0": (_i, [_vp, _vp, _sz, _vp, _vp]),
    "dk_q8_0_group_dots": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "dk_q8_row_bytes": (_sz, [_i]),
    "dk_q8_tile_rows": (_i, [_i]),
    "dk_q8_packed_bytes": (_sz, [_i, _i]),
    "dk_q8_pack": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "dk_matmul_q8_0": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "dk_matmul_q8_0_q": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "dk_matmul_q8_0_batch": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "dk_matmul_q8_0_tokens": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "dk_sample": (_i, [_vp, _i, C.c_float, C.c_float, C.c_float, _vp, _vp, _vp]),
    "dk_softmax": (_i, [_vp, _i, _vp]),
    "dk_rmsnorm": (_i, [_vp, _vp, _vp, _i, _vp]),
    "dk_attention_work_bytes": (_sz, [_i, _i, _i, _i]),
    "dk_attention_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _vp, _vp]),
    "dk_attention_decode_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _vp]),
    "dk_model_create": (_vp, [C.POINTER(C.c_int), _i, _i, _i, _i]),
    "dk_model_destroy": (None, [_vp]),
    "dk_model_set_weight": (_i, [_vp, _i, _i, _vp, _vp]),
    "dk_model_set_weight_device": (_i, [_vp, _i, _i, _vp, _vp]),
    "dk_model_comm_handle": (_i, [_vp, _vp]),
    "dk_model_comm_connect": (_i, [_vp, _vp]),
    "dk_model_finalize": (_i, [_vp]),
    "dk_model_forward": (_i, [_vp, _i, _i, _vp]),
    "dk_model_generate": (_i, [_vp, _vp, _i, _i, _vp, C.POINTER(C.c_int)]),
    "dk_model_set_tokens": (_i, [_vp, _vp, _i, _i]),
    "dk_model_enqueue_steps": (_i, [_vp, _i, _i]),
    "dk_model_prefill": (_i, [_vp, _i, _i]),
    "dk_gemm_trace": (_i, [_vp, _sz, _vp, _vp]),
    "dk_attn_split_plan": (_i, [_i, _i, _i, _vp, _vp]),
    "dk_step_attn_plan": (_i, [_i, _vp, _vp, _vp]),
    "dk_prefill_attn_plan": (_i, [_i, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "dk_model_get_tokens": (_i, [_vp, _vp, _i]),
    "dk_model_sync": (_i, [_vp]),
    "dk_model_stream": (_vp, [_vp]),
    "dk_model_device_error": (_i, [_vp]),
    "dk_model_kernels_per_step": (_i, [_vp]),
    "dk_model_weight_bytes": (_sz, [_vp]),
    "dk_model_trace": (_i, [_vp, _vp, _sz, _vp, _vp]),
    "dk_model_dump_enable": (_i, [_vp, _i]),
    "dk_model_dump_read": (_i, [_vp, _vp, _vp, _vp]),
    "dk_model_kv_write": (_i, [_vp, _i, _i, _i, _vp, _vp, _i]),
    "dk_model_kv_read": (_i, [_vp, _i, _i, _i, _vp, _vp]),
}

_lib = None


class DiolkosError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"diolkos error 0x{code:x}: {msg}")
        self.code = code


def lib() -> C.CDLL:
    """The loaded library (built by diolkos_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m diolkos_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(code: int) -> None:
    if code != DK_OK:
        msg = lib().dk_last_error()
        raise DiolkosError(code, msg.decode() if msg else "")


def stream_ptr(stream=None) -> int | None:
    """cudaStream_t of a torch stream (None -> the current torch stream)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
