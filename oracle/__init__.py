"""The oracle: ctypes bindings to the CPU restatement (port.c) and to the compiled reference.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline
leg import this package, and only as the checker; the product (``diolkos_b200``) never does.

* :class:`Port` wraps ``oracle/liboracle_port.so`` (the restatement; always built).
* :class:`Ref` wraps ``oracle/_ref/<variant>/liboracle_ref.so`` (the unmodified reference sources
  compiled with the reference's flags; built only where the reference tree is present, then
  carried along with the working tree).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle_port.so")
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

PW_EMB, PW_RMS_FINAL, PW_WCLS, PW_RMS_ATT, PW_WQ, PW_WK, PW_WV, PW_WO, PW_RMS_FFN, PW_W1, PW_W2, PW_W3 = range(12)


class Port:
    """The restatement in port.c."""

    def __init__(self, path: str = PORT_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built; run `make -C oracle port`")
        L = self.lib = C.CDLL(path)
        L.port_quant_bf16.argtypes = [_u16p, C.c_size_t, _i8p, _f32p]
        L.port_quant_f32.argtypes = [_f32p, C.c_size_t, _i8p, _f32p]
        L.port_dequant.argtypes = [_i8p, _f32p, C.c_size_t, _f32p]
        L.port_matmul.argtypes = [_f32p, _f32p, _i8p, _f32p, C.c_int, C.c_int]
        L.port_matmul_q.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, C.c_int, C.c_int]
        L.port_group_dots.argtypes = [_i32p, _i8p, _i8p, C.c_int, C.c_int]
        L.port_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        L.port_softmax.argtypes = [_f32p, C.c_int]
        L.port_argmax.argtypes = [_f32p, C.c_int]
        L.port_argmax.restype = C.c_int
        L.port_rope_coeffs.argtypes = [C.c_int, C.c_int, _f32p]
        L.port_sample.argtypes = [_f32p, C.c_int, C.c_float, C.c_float, C.POINTER(C.c_ulonglong)]
        L.port_sample.restype = C.c_int
        L.port_model_create.argtypes = [_i32p, C.c_int]
        L.port_model_create.restype = C.c_void_p
        L.port_model_destroy.argtypes = [C.c_void_p]
        L.port_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.port_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_void_p]
        L.port_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p]
        L.port_forward_dump.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p, _f32p, _i8p, _f32p]
        L.port_kv_rows.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.port_kv_write.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.port_generate.restype = C.c_int

    def quant_bf16(self, x_bits: np.ndarray):
        x = np.ascontiguousarray(x_bits, dtype=np.uint16).ravel()
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // 32, np.float32)
        self.lib.port_quant_bf16(x, x.size, q, s)
        return q, s

    def quant_f32(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // 32, np.float32)
        self.lib.port_quant_f32(x, x.size, q, s)
        return q, s

    def dequant(self, q, s):
        out = np.empty(q.size, np.float32)
        self.lib.port_dequant(np.ascontiguousarray(q, np.int8).ravel(),
                              np.ascontiguousarray(s, np.float32).ravel(), q.size, out)
        return out

    def matmul(self, x, wq, ws, n, d):
        out = np.empty(d, np.float32)
        self.lib.port_matmul(out, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(wq, np.int8).ravel(),
                             np.ascontiguousarray(ws, np.float32).ravel(), n, d)
        return out

    def matmul_q(self, xq, xs, wq, ws, n, d):
        out = np.empty(d, np.float32)
        self.lib.port_matmul_q(out, np.ascontiguousarray(xq, np.int8), np.ascontiguousarray(xs, np.float32),
                               np.ascontiguousarray(wq, np.int8).ravel(),
                               np.ascontiguousarray(ws, np.float32).ravel(), n, d)
        return out

    def group_dots(self, xq, wq, n, d):
        dots = np.empty((d, n // 32), np.int32)
        self.lib.port_group_dots(dots, np.ascontiguousarray(xq, np.int8),
                                 np.ascontiguousarray(wq, np.int8).ravel(), n, d)
        return dots

    def rmsnorm(self, x, w):
        o = np.empty(x.size, np.float32)
        self.lib.port_rmsnorm(o, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32), x.size)
        return o

    def softmax(self, x):
        y = np.array(x, dtype=np.float32, copy=True)
        self.lib.port_softmax(y, y.size)
        return y

    def argmax(self, x):
        return int(self.lib.port_argmax(np.ascontiguousarray(x, np.float32), x.size))

    def rope_coeffs(self, pos, head_size):
        cs = np.empty(head_size, np.float32)
        self.lib.port_rope_coeffs(pos, head_size, cs)
        return cs

    def sample(self, logits, temperature, topp, rng_state):
        y = np.array(logits, dtype=np.float32, copy=True)
        st = C.c_ulonglong(rng_state)
        tok = self.lib.port_sample(y, y.size, temperature, topp, C.byref(st))
        return int(tok), int(st.value)


class PortModel:
    """A whole model in the restatement; holds references to the weight arrays it registers."""

    def __init__(self, port: Port, cfg, weights: dict, kv_f32: bool = False):
        self.port, self.cfg, self.kv_f32 = port, cfg, kv_f32
        self._keep = []
        self.h = port.lib.port_model_create(np.array(cfg.as_list(), np.int32), int(kv_f32))
        for (which, layer), w in weights.items():
            if isinstance(w, tuple):
                q = np.ascontiguousarray(w[0], np.int8)
                s = np.ascontiguousarray(w[1], np.float32)
                self._keep += [q, s]
                port.lib.port_model_set(self.h, which, layer, q.ctypes.data, s.ctypes.data)
            else:
                v = np.ascontiguousarray(w, np.float32)
                self._keep.append(v)
                port.lib.port_model_set(self.h, which, layer, v.ctypes.data, None)

    def forward(self, token, pos, dump_layers=False):
        logits = np.empty(self.cfg.vocab_size, np.float32)
        xd = np.empty((self.cfg.n_layers, self.cfg.dim), np.float32) if dump_layers else None
        self.port.lib.port_forward(self.h, token, pos, logits, xd.ctypes.data if xd is not None else None)
        return (logits, xd) if dump_layers else logits

    def generate(self, prompt, steps):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(max(steps, 1), np.int32)
        n = self.port.lib.port_generate(self.h, p, p.size, steps, out)
        return out[:n].copy()

    def forward_dump(self, token, pos):
        """forward with per-layer checkpoints, the layout of RefModel.forward_dump."""
        c = self.cfg
        sizes = [c.dim, c.dim, c.dim, c.hidden_dim] * c.n_layers + [c.dim]
        tot = sum(sizes)
        logits = np.empty(c.vocab_size, np.float32)
        xres = np.empty((2 * c.n_layers + 1, c.dim), np.float32)
        ain, aq, asc = np.empty(tot, np.float32), np.empty(tot, np.int8), np.empty(tot // 32, np.float32)
        self.port.lib.port_forward_dump(self.h, token, pos, logits, xres, ain, aq, asc)
        acts, off = [], 0
        for n in sizes:
            acts.append((ain[off:off + n], aq[off:off + n], asc[off // 32:(off + n) // 32]))
            off += n
        return logits, xres, acts

    def kv_write(self, layer, pos0, k, v):
        """Overwrite KV-cache rows pos0.. of one layer ([n][kv_dim] of the cache's element type)."""
        k = np.ascontiguousarray(k)
        v = np.ascontiguousarray(v)
        kv_dim = self.cfg.dim * self.cfg.n_kv_heads // self.cfg.n_heads
        self.port.lib.port_kv_write(self.h, layer, pos0, k.size // kv_dim, k.ctypes.data, v.ctypes.data)

    def kv_rows(self, layer, pos0, n):
        """KV-cache rows of positions pos0 .. pos0+n-1 ([n][kv_dim]): uint16 bf16 bits, or float32 for an
        fp32 cache."""
        c = self.cfg
        kv_dim = c.dim * c.n_kv_heads // c.n_heads
        dt = np.float32 if self.kv_f32 else np.uint16
        k, v = np.empty((n, kv_dim), dt), np.empty((n, kv_dim), dt)
        self.port.lib.port_kv_rows(self.h, layer, pos0, n, k.ctypes.data, v.ctypes.data)
        return k, v

    def __del__(self):
        try:
            self.port.lib.port_model_destroy(self.h)
        except Exception:
            pass


def ref_path(variant: str = "auto", hooked: bool = False) -> str | None:
    """Path of the compiled reference library, or None when it was not built here.

    "auto" prefers the portable (-march=x86-64-v3) build: its arithmetic is the same on every
    AVX2+FMA host, whereas -march=native lets the compiler pick a host-dependent vector shape that
    changes the order of the GEMV's fp32 sums.  hooked: the build whose forward() records per-layer
    checkpoints (ref_hooks.c; portable only)."""
    order = ["portable", "native"] if variant == "auto" else [variant]
    name = "liboracle_ref_hooked.so" if hooked else "liboracle_ref.so"
    for v in order:
        p = os.path.join(REF_DIR, v, name)
        if os.path.exists(p):
            return p
    return None


class Ref:
    """The unmodified reference C code (oracle/_ref), driven through ref_driver.c."""

    def __init__(self, variant: str = "auto", hooked: bool = False):
        p = ref_path(variant, hooked)
        if p is None:
            raise FileNotFoundError("oracle/_ref is not built (needs the reference source tree)")
        self.path, self.hooked = p, hooked
        L = self.lib = C.CDLL(p)
        if hooked:
            L.oref_forward_dump.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p, _f32p, _i8p, _f32p, _i32p]
        L.oref_load.argtypes = [C.c_char_p, C.c_char_p]
        L.oref_load.restype = C.c_void_p
        L.oref_config.argtypes = [C.c_void_p, _i32p]
        L.oref_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
        L.oref_state_x.argtypes = [C.c_void_p, _f32p]
        L.oref_kv_rows.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _u16p, _u16p]
        L.oref_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p, C.POINTER(C.c_double),
                                    C.POINTER(C.c_double), C.c_void_p]
        L.oref_threads.argtypes = [C.c_int]
        L.oref_threads.restype = C.c_int
        L.oref_generate.restype = C.c_int
        L.oref_quant_f32.argtypes = [_f32p, C.c_size_t, _i8p, _f32p]
        L.oref_quant_bf16.argtypes = [_u16p, C.c_size_t, _i8p, _f32p]
        L.oref_mat_create.argtypes = [_i8p, _f32p, C.c_int, C.c_int]
        L.oref_mat_create.restype = C.c_void_p
        L.oref_mat_run.argtypes = [C.c_void_p, _f32p, _f32p]
        L.oref_mat_time.argtypes = [C.c_void_p, C.c_int]
        L.oref_mat_time.restype = C.c_double
        L.oref_mat_destroy.argtypes = [C.c_void_p]
        L.oref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        L.oref_softmax.argtypes = [_f32p, C.c_int]
        L.oref_argmax.argtypes = [_f32p, C.c_int]
        L.oref_argmax.restype = C.c_int
        L.oref_sample.argtypes = [_f32p, C.c_int, C.c_float, C.c_float, C.POINTER(C.c_ulonglong)]
        L.oref_sample.restype = C.c_int

    def threads(self, n: int = 0) -> int:
        """Set (n > 0) and return the OpenMP thread count of the reference's parallel loops."""
        return int(self.lib.oref_threads(n))

    def quant_f32(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // 32, np.float32)
        self.lib.oref_quant_f32(x, x.size, q, s)
        return q, s

    def quant_bf16(self, x_bits):
        x = np.ascontiguousarray(x_bits, np.uint16).ravel()
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // 32, np.float32)
        self.lib.oref_quant_bf16(x, x.size, q, s)
        return q, s

    def matmul(self, x, wq, ws, n, d):
        m = self.lib.oref_mat_create(np.ascontiguousarray(wq, np.int8).ravel(),
                                     np.ascontiguousarray(ws, np.float32).ravel(), n, d)
        out = np.empty(d, np.float32)
        self.lib.oref_mat_run(m, np.ascontiguousarray(x, np.float32), out)
        self.lib.oref_mat_destroy(m)
        return out

    def rmsnorm(self, x, w):
        o = np.empty(x.size, np.float32)
        self.lib.oref_rmsnorm(o, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32), x.size)
        return o

    def softmax(self, x):
        y = np.array(x, dtype=np.float32, copy=True)
        self.lib.oref_softmax(y, y.size)
        return y

    def argmax(self, x):
        return int(self.lib.oref_argmax(np.ascontiguousarray(x, np.float32), x.size))

    def sample(self, logits, temperature, topp, rng_state):
        y = np.array(logits, dtype=np.float32, copy=True)
        st = C.c_ulonglong(rng_state)
        tok = self.lib.oref_sample(y, y.size, temperature, topp, C.byref(st))
        return int(tok), int(st.value)

    def load(self, model_dir: str, work_dir: str):
        h = self.lib.oref_load(os.path.abspath(model_dir).encode(), os.path.abspath(work_dir).encode())
        if not h:
            raise RuntimeError("reference load failed")
        return RefModel(self, h)


class RefModel:
    def __init__(self, ref: Ref, h):
        self.ref, self.h = ref, h
        cfg = np.empty(7, np.int32)
        ref.lib.oref_config(h, cfg)
        self.cfg = [int(v) for v in cfg]

    def forward(self, token, pos):
        logits = np.empty(self.cfg[5], np.float32)
        self.ref.lib.oref_forward(self.h, token, pos, logits)
        return logits

    def generate(self, prompt, steps):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(max(steps, 1), np.int32)
        tps = C.c_double(0.0)
        n = self.ref.lib.oref_generate(self.h, p, p.size, steps, out, C.byref(tps), None, None)
        return out[:n].copy(), tps.value

    def generate_timed(self, prompt, steps):
        """The reference's generate loop: (generated tokens, wall seconds of the positions that produced
        them, top-2 logits per generated token [n][2])."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(max(steps, 1), np.int32)
        top2 = np.empty((max(steps, 1), 2), np.float32)
        tps, gs = C.c_double(0.0), C.c_double(0.0)
        n = self.ref.lib.oref_generate(self.h, p, p.size, steps, out, C.byref(tps), C.byref(gs), top2.ctypes.data)
        return out[:n].copy(), gs.value, top2[:n].copy()

    def kv_rows(self, layer, pos0, n):
        """The reference's bf16 KV-cache rows (uint16 bits) of positions pos0 .. pos0+n-1: (k, v), [n][kv_dim]."""
        kv_dim = self.cfg[0] * self.cfg[4] // self.cfg[3]
        k = np.empty((n, kv_dim), np.uint16)
        v = np.empty((n, kv_dim), np.uint16)
        self.ref.lib.oref_kv_rows(self.h, layer, pos0, n, k, v)
        return k, v

    def forward_dump(self, token, pos):
        """forward() with per-layer checkpoints (hooked build only).  Returns (logits, xres, acts):
        xres[2L+1][dim] = the residual stream before each rmsnorm (the embedding row, then x after every
        residual add); acts = per layer [attention-norm input activation, attention output, FFN-norm
        output, SwiGLU output] then the classifier's: each (fp32 input, int8 Q8_0 values, fp32 scales)
        exactly as matmul_Q8_0 quantised it."""
        if not self.ref.hooked:
            raise RuntimeError("forward_dump needs Ref(hooked=True)")
        dim, hidden, L, vocab = self.cfg[0], self.cfg[1], self.cfg[2], self.cfg[5]
        sizes = [dim, dim, dim, hidden] * L + [dim]
        tot = sum(sizes)
        logits = np.empty(vocab, np.float32)
        xres = np.empty((2 * L + 1, dim), np.float32)
        ain = np.empty(tot, np.float32)
        aq = np.empty(tot, np.int8)
        asc = np.empty(tot // 32, np.float32)
        counts = np.zeros(2, np.int32)
        self.ref.lib.oref_forward_dump(self.h, token, pos, logits, xres, ain, aq, asc, counts)
        if counts[0] != 2 * L + 1 or counts[1] != 7 * L + 1:
            raise RuntimeError(f"hooked forward made {counts[0]} rmsnorm / {counts[1]} matmul calls")
        acts, off = [], 0
        for n in sizes:
            acts.append((ain[off:off + n], aq[off:off + n], asc[off // 32:(off + n) // 32]))
            off += n
        return logits, xres, acts


def load_port_weights(port: Port, cfg, seed: int):
    """Regenerate a seeded synthetic model (diolkos_b200.synth) and quantise it with the
    restatement's load-time quantiser; returns the dict PortModel expects plus the raw Q8 arrays
    keyed by HF tensor name."""
    from diolkos_b200 import synth

    names = {
        "input_layernorm.weight": PW_RMS_ATT, "self_attn.q_proj.weight": PW_WQ,
        "self_attn.k_proj.weight": PW_WK, "self_attn.v_proj.weight": PW_WV,
        "self_attn.o_proj.weight": PW_WO, "post_attention_layernorm.weight": PW_RMS_FFN,
        "mlp.gate_proj.weight": PW_W1, "mlp.down_proj.weight": PW_W2, "mlp.up_proj.weight": PW_W3,
    }
    weights, by_name = {}, {}
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        bits = synth.gen_tensor(seed, idx, kind, shape)
        if kind == "q8":
            val = port.quant_bf16(bits)
        else:
            val = synth.bf16_bits_to_f32(bits)
        by_name[name] = val
        if name == "model.embed_tokens.weight":
            key = (PW_EMB, -1)
        elif name == "lm_head.weight":
            key = (PW_WCLS, -1)
        elif name == "model.norm.weight":
            key = (PW_RMS_FINAL, -1)
        else:
            rest = name[len("model.layers."):]
            layer, suffix = rest.split(".", 1)
            key = (names[suffix], int(layer))
        weights[key] = val
    return weights, by_name
