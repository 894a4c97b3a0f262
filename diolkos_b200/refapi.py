"""ctypes mirror of the reference-compatible C API that libdiolkos.so exports (include/tensor.h,
transformer.h, safetensors.h, utils.h, sampler.h, tokenizer.h).

The structures have the reference's layouts exactly (src/tensor.h:18-28, src/transformer.h:14-51,
src/safetensors.h:11-33, src/sampler.h:4-16, src/tokenizer.h:5-20).  These entry points keep the reference's failure behaviour: a
bad input prints a message and exits the process, so call them only with inputs that are known to
be valid (or from a child process).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native

F32, F16, BF16, Q8_0, Q4_0 = range(5)


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int), ("data", C.c_void_p), ("scale", C.POINTER(C.c_float)), ("dim", C.c_size_t),
                ("hdim", C.c_size_t), ("vdim", C.c_size_t), ("tensor_id", C.c_uint32), ("fd", C.c_int)]

    def f32(self) -> np.ndarray:
        assert self.type == F32
        return np.ctypeslib.as_array(C.cast(self.data, C.POINTER(C.c_float)), shape=(self.dim,)).copy()

    def q8(self) -> tuple[np.ndarray, np.ndarray]:
        assert self.type == Q8_0
        q = np.ctypeslib.as_array(C.cast(self.data, C.POINTER(C.c_int8)), shape=(self.dim,)).copy()
        s = np.ctypeslib.as_array(self.scale, shape=(self.dim // 32,)).copy()
        return q, s


TensorP = C.POINTER(Tensor)


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                                       "seq_len")]


class RunState(C.Structure):
    _fields_ = [(n, TensorP) for n in ("x", "xb", "xb2", "hb", "hb2", "q", "att", "logits", "key_cache",
                                       "value_cache", "k", "v")]


class Layer(C.Structure):
    _fields_ = [(n, TensorP) for n in ("rms_att_weight", "rms_ffn_weight", "wq", "wk", "wv", "wo", "w1", "w2",
                                       "w3")]


class Model(C.Structure):
    _fields_ = [("config", C.POINTER(Config)), ("huggingface_rope", C.c_bool),
                ("token_embedding_table", TensorP), ("layers", C.POINTER(Layer)),
                ("rms_final_weight", TensorP), ("wcls", TensorP)]


class Transformer(C.Structure):
    _fields_ = [("config", Config), ("state", RunState), ("safetensors", C.POINTER(Model))]


class ProbIndex(C.Structure):
    _fields_ = [("prob", C.c_float), ("index", C.c_int)]


class Sampler(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("probindex", C.POINTER(ProbIndex)), ("temperature", C.c_float),
                ("topp", C.c_float), ("rng_state", C.c_ulonglong)]


class TokenIndex(C.Structure):
    _fields_ = [("str", C.c_char_p), ("id", C.c_int)]


class Tokenizer(C.Structure):
    _fields_ = [("vocab", C.POINTER(C.c_char_p)), ("vocab_scores", C.POINTER(C.c_float)),
                ("sorted_vocab", C.POINTER(TokenIndex)), ("vocab_size", C.c_int), ("max_token_length", C.c_uint),
                ("byte_pieces", C.c_ubyte * 512), ("bos_id", C.c_int), ("eos_id", C.c_int)]


_SIGS = {
    "bf16_to_float": (C.c_float, [C.c_uint16]),
    "f16_to_float": (C.c_float, [C.c_uint16]),
    "tensor_create": (TensorP, [C.c_size_t, C.c_int]),
    "tensor_destroy": (None, [TensorP]),
    "Tensor_storage_size": (C.c_size_t, [TensorP]),
    "tensor_memory": (C.c_size_t, [TensorP]),
    "convert": (TensorP, [TensorP, C.c_int]),
    "data_f32": (C.POINTER(C.c_float), [TensorP]),
    "data_i8": (C.POINTER(C.c_int8), [TensorP]),
    "group_size": (C.c_int, [C.c_int]),
    "quant_size": (C.c_int, [C.c_int]),
    "quant_t_to_string": (C.c_char_p, [C.c_int]),
    "reliable_isnan": (C.c_bool, [C.c_double]),
    "round_down_32": (C.c_size_t, [C.c_size_t]),
    "softmax": (None, [TensorP, C.c_int]),
    "softmax_f32": (None, [C.POINTER(C.c_float), C.c_int]),
    "rmsnorm": (None, [TensorP, TensorP, TensorP, C.c_int]),
    "matmul": (None, [TensorP, TensorP, TensorP, C.c_int, C.c_int]),
    "init_utils": (None, [C.c_int, C.c_int]),
    "malloc_run_state": (None, [C.POINTER(RunState), C.POINTER(Config)]),
    "build_transformer_from_safetensors": (None, [C.POINTER(Transformer), C.c_char_p]),
    "forward": (TensorP, [C.POINTER(Transformer), C.c_int, C.c_int]),
    "free_transformer": (None, [C.POINTER(Transformer)]),
    "transformer_engine": (C.c_void_p, [C.POINTER(Transformer)]),
    "load_safetensors": (C.POINTER(Model), [C.c_char_p]),
    "build_sampler": (None, [C.POINTER(Sampler), C.c_int, C.c_float, C.c_float, C.c_ulonglong]),
    "free_sampler": (None, [C.POINTER(Sampler)]),
    "sample": (C.c_int, [C.POINTER(Sampler), C.POINTER(C.c_float)]),
    "random_u32": (C.c_uint, [C.POINTER(C.c_ulonglong)]),
    "random_f32": (C.c_float, [C.POINTER(C.c_ulonglong)]),
    "build_tokenizer": (None, [C.POINTER(Tokenizer), C.c_char_p]),
    "free_tokenizer": (None, [C.POINTER(Tokenizer)]),
    "decode": (C.c_void_p, [C.POINTER(Tokenizer), C.c_int, C.c_int]),
    "safe_printf": (None, [C.c_char_p]),
    "encode": (None, [C.POINTER(Tokenizer), C.c_char_p, C.c_int8, C.c_int8, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "str_lookup": (C.c_int, [C.c_char_p, C.POINTER(TokenIndex), C.c_int]),
}


def bind(lib: C.CDLL, names=None) -> C.CDLL:
    """Set restype/argtypes of the reference-API functions on `lib` (libdiolkos.so, or any library
    that exports the same API)."""
    for name, (res, args) in _SIGS.items():
        if names is not None and name not in names:
            continue
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


_bound = None


def lib() -> C.CDLL:
    """libdiolkos.so with the reference-API signatures set."""
    global _bound
    if _bound is None:
        _bound = bind(_native.lib())
    return _bound


# ---- convenience wrappers --------------------------------------------------------------------
def encode(tok: Tokenizer, text: bytes, bos: bool = True, eos: bool = False, L: C.CDLL | None = None) -> list[int]:
    L = L or lib()
    buf = (C.c_int * (len(text) + 3))()
    n = C.c_int(0)
    L.encode(C.byref(tok), text, 1 if bos else 0, 1 if eos else 0, buf, C.byref(n))
    return list(buf[: n.value])


def decode(tok: Tokenizer, prev: int, token: int, L: C.CDLL | None = None) -> bytes:
    L = L or lib()
    return C.string_at(L.decode(C.byref(tok), prev, token))


def load_tokenizer(path: str, L: C.CDLL | None = None) -> Tokenizer:
    L = L or lib()
    tok = Tokenizer()
    L.build_tokenizer(C.byref(tok), path.encode())
    return tok
