"""Python mirror of the decode engine (dk_model_* in include/diolkos.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from . import synth

# HF tensor name suffix -> weight id
_LAYER_IDS = {
    "input_layernorm.weight": N.DK_W_RMS_ATT, "self_attn.q_proj.weight": N.DK_W_WQ,
    "self_attn.k_proj.weight": N.DK_W_WK, "self_attn.v_proj.weight": N.DK_W_WV,
    "self_attn.o_proj.weight": N.DK_W_WO, "post_attention_layernorm.weight": N.DK_W_RMS_FFN,
    "mlp.gate_proj.weight": N.DK_W_W1, "mlp.down_proj.weight": N.DK_W_W2, "mlp.up_proj.weight": N.DK_W_W3,
}


def weight_id(name: str) -> tuple[int, int]:
    """(weight id, layer) of an HF tensor name."""
    if name == "model.embed_tokens.weight":
        return N.DK_W_EMB, -1
    if name == "lm_head.weight":
        return N.DK_W_WCLS, -1
    if name == "model.norm.weight":
        return N.DK_W_RMS_FINAL, -1
    rest = name[len("model.layers."):]
    layer, suffix = rest.split(".", 1)
    return _LAYER_IDS[suffix], int(layer)


class Model:
    """One model resident on one GPU; the whole decode step is a CUDA graph."""

    def __init__(self, cfg: synth.Config, kv_f32: bool = False, device: int = 0, tp_rank: int = 0,
                 tp_world: int = 1):
        self.cfg = cfg
        self.kv_f32 = kv_f32
        self.tp_rank, self.tp_world = tp_rank, tp_world
        L = N.lib()
        arr = (C.c_int * 7)(*cfg.as_list())
        self.h = L.dk_model_create(arr, N.DK_KV_F32 if kv_f32 else N.DK_KV_BF16, device, tp_rank, tp_world)
        if not self.h:
            raise N.DiolkosError(N.DK_ERR_INVALID, L.dk_last_error().decode())

    def comm_handle(self) -> bytes:
        """This rank's exchange-area IPC handle (tensor parallel)."""
        buf = C.create_string_buffer(N.DK_COMM_HANDLE_BYTES)
        N.check(N.lib().dk_model_comm_handle(self.h, buf))
        return buf.raw

    def comm_connect(self, handles: list) -> None:
        """Map every rank's exchange area (handles in rank order, this rank's included)."""
        blob = b"".join(handles)
        if len(blob) != N.DK_COMM_HANDLE_BYTES * self.tp_world:
            raise ValueError("one handle per rank expected")
        buf = C.create_string_buffer(blob, len(blob))
        N.check(N.lib().dk_model_comm_connect(self.h, buf))

    def set_weight(self, which: int, layer: int, q, s=None):
        """Host arrays: Q8_0 (int8 q, fp32 s) planar, or a fp32 vector."""
        q = np.ascontiguousarray(q)
        if s is not None:
            s = np.ascontiguousarray(s, dtype=np.float32)
        N.check(N.lib().dk_model_set_weight(self.h, which, layer, q.ctypes.data,
                                             s.ctypes.data if s is not None else None))

    def set_weight_device(self, which: int, layer: int, q, s=None):
        """Device tensors (torch): Q8_0 planar (int8, fp32) or a fp32 vector.  The engine copies on its
        own stream, so the torch stream that produced the tensors is synchronised first."""
        import torch

        torch.cuda.current_stream(q.device).synchronize()
        N.check(N.lib().dk_model_set_weight_device(self.h, which, layer, q.data_ptr(),
                                                    s.data_ptr() if s is not None else None))

    def load_named(self, weights_by_name: dict):
        for name, val in weights_by_name.items():
            which, layer = weight_id(name)
            if isinstance(val, tuple):
                self.set_weight(which, layer, val[0], val[1])
            else:
                self.set_weight(which, layer, np.asarray(val, dtype=np.float32))

    def finalize(self):
        N.check(N.lib().dk_model_finalize(self.h))

    def forward(self, token: int, pos: int) -> np.ndarray:
        """Logits of one step (tensor parallel: only this rank's classifier rows are filled, the rest
        is NaN)."""
        logits = np.full(self.cfg.vocab_size, np.nan, np.float32)
        N.check(N.lib().dk_model_forward(self.h, token, pos, logits.ctypes.data))
        return logits

    def generate(self, prompt, steps: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max(steps, 1), np.int32)
        n = C.c_int(0)
        N.check(N.lib().dk_model_generate(self.h, p.ctypes.data, p.size, steps, out.ctypes.data, C.byref(n)))
        return out[: n.value].copy()

    def set_tokens(self, tokens, n_forced: int):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        N.check(N.lib().dk_model_set_tokens(self.h, t.ctypes.data, t.size, n_forced))

    def enqueue_steps(self, pos0: int, n_steps: int):
        N.check(N.lib().dk_model_enqueue_steps(self.h, pos0, n_steps))

    def prefill(self, pos0: int, n_positions: int):
        """Batched prefill of prompt positions [pos0, pos0 + n_positions) on the tensor cores (tokens
        from set_tokens); fills their KV-cache entries, enqueued."""
        N.check(N.lib().dk_model_prefill(self.h, pos0, n_positions))

    def get_tokens(self, n: int) -> np.ndarray:
        t = np.empty(n, np.int32)
        N.check(N.lib().dk_model_get_tokens(self.h, t.ctypes.data, n))
        return t

    def sync(self):
        N.check(N.lib().dk_model_sync(self.h))

    @property
    def stream(self) -> int:
        return N.lib().dk_model_stream(self.h)

    def device_error(self) -> int:
        return N.lib().dk_model_device_error(self.h)

    def dump_enable(self, on: bool = True) -> None:
        """Record every later decode step's per-op inputs and Q8_0 activations (dk_model_dump_enable)."""
        N.check(N.lib().dk_model_dump_enable(self.h, int(on)))

    def kv_write(self, layer: int, pos0: int, k, v) -> None:
        """Overwrite KV rows pos0.. of one layer with rows in the reference's layout ([n][kv_dim]):
        uint16 arrays are bf16 bits, float32 arrays fp32 values."""
        k = np.ascontiguousarray(k)
        v = np.ascontiguousarray(v)
        if k.dtype == np.uint16:
            t = N.DK_KV_BF16
        elif k.dtype == np.float32:
            t = N.DK_KV_F32
        else:
            raise TypeError("KV rows must be uint16 (bf16 bits) or float32")
        kv_dim = self.cfg.n_kv_heads * (self.cfg.dim // self.cfg.n_heads)
        N.check(N.lib().dk_model_kv_write(self.h, layer, pos0, k.size // kv_dim, k.ctypes.data, v.ctypes.data, t))

    def kv_read(self, layer: int, pos0: int, n: int = 1):
        """This rank's KV rows pos0 .. pos0+n-1 of one layer ([n][kv_dim]; uint16 bf16 bits, or float32
        for an fp32 cache)."""
        kv_dim = (self.cfg.n_kv_heads // self.tp_world) * (self.cfg.dim // self.cfg.n_heads)
        dt = np.float32 if self.kv_f32 else np.uint16
        k, v = np.empty((n, kv_dim), dt), np.empty((n, kv_dim), dt)
        N.check(N.lib().dk_model_kv_read(self.h, layer, pos0, n, k.ctypes.data, v.ctypes.data))
        return k, v

    def dump_read(self):
        """The last step's record: per layer [q|k|v input, wo input, w1|w3 input, w2 input], then the
        classifier's; each (fp32 input, int8 values, fp32 scales).  Under tensor parallelism the wo and
        w2 inputs are this rank's slices (its heads' attention output, its SwiGLU rows)."""
        c = self.cfg
        W = self.tp_world
        sizes = [c.dim, c.dim // W, c.dim, c.hidden_dim // W] * c.n_layers + [c.dim]
        tot = sum(sizes)
        ain = np.empty(tot, np.float32)
        aq = np.empty(tot, np.int8)
        asc = np.empty(tot // 32, np.float32)
        N.check(N.lib().dk_model_dump_read(self.h, ain.ctypes.data, aq.ctypes.data, asc.ctypes.data))
        out, off = [], 0
        for n in sizes:
            out.append((ain[off:off + n], aq[off:off + n], asc[off // 32:(off + n) // 32]))
            off += n
        return out

    @property
    def kernels_per_step(self) -> int:
        return N.lib().dk_model_kernels_per_step(self.h)

    @property
    def weight_bytes(self) -> int:
        return int(N.lib().dk_model_weight_bytes(self.h))

    def close(self):
        if getattr(self, "h", None):
            N.lib().dk_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
