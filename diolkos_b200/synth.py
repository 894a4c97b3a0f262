"""Seeded synthetic LLaMA-2 checkpoints in the formats the Diolkos loader reads.

Writes what ``load_safetensors`` (reference src/safetensors.c:275-405) consumes:

* ``config.json`` with the HF keys the reference reads (src/safetensors.c:293-299);
* ``model.safetensors``: an 8-byte little-endian header length, a JSON header, then the raw
  tensor bytes (src/safetensors.c:151-161), all tensors BF16 with HF names
  (src/safetensors.c:166-266);
* optionally a *header-only* safetensors plus pre-written Q8_0 cache files
  ``cache/<model>/<tensor>-Q8_0.tensor`` (int8[n] then fp32[n/32], src/safetensors.c:57-114) and
  ``-F32.tensor`` for the norms, which the reference and this library load without reading any
  tensor data (used for models too large to write as bf16);
* a ``tokenizer.bin`` in the llama2.c layout (src/tokenizer.c:11-48) with a " " piece.

Weights are N(0, 0.02) drawn in fp32 from numpy's PCG64 seeded with ``(seed, tensor_index)`` and
rounded to bf16 (round-to-nearest-even); RMSNorm weights are 1.0.  The same seed gives the same
bytes on every machine, so a model can be regenerated wherever a test runs.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, asdict

import numpy as np


@dataclass(frozen=True)
class Config:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int

    @property
    def head_size(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.dim * self.n_kv_heads // self.n_heads

    def as_list(self) -> list[int]:
        return [self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
                self.vocab_size, self.seq_len]

    def replace(self, **kw) -> "Config":
        d = asdict(self)
        d.update(kw)
        return Config(**d)


# The model shapes the benchmarks and parity tests use.
TINY = Config(288, 768, 6, 6, 6, 32000, 256)
LLAMA7B = Config(4096, 11008, 32, 32, 32, 32000, 4096)
LLAMA70B = Config(8192, 28672, 80, 64, 8, 32000, 4096)

# Per-layer tensor names in HF LLaMA checkpoints, with (rows, cols) as functions of the config.
LAYER_TENSORS = [
    ("input_layernorm.weight", "norm", lambda c: (c.dim,)),
    ("self_attn.q_proj.weight", "q8", lambda c: (c.n_heads * c.head_size, c.dim)),
    ("self_attn.k_proj.weight", "q8", lambda c: (c.kv_dim, c.dim)),
    ("self_attn.v_proj.weight", "q8", lambda c: (c.kv_dim, c.dim)),
    ("self_attn.o_proj.weight", "q8", lambda c: (c.dim, c.n_heads * c.head_size)),
    ("post_attention_layernorm.weight", "norm", lambda c: (c.dim,)),
    ("mlp.gate_proj.weight", "q8", lambda c: (c.hidden_dim, c.dim)),
    ("mlp.down_proj.weight", "q8", lambda c: (c.dim, c.hidden_dim)),
    ("mlp.up_proj.weight", "q8", lambda c: (c.hidden_dim, c.dim)),
]


def tensor_specs(cfg: Config) -> list[tuple[str, str, tuple[int, ...]]]:
    """(name, kind, shape) for every tensor, in a fixed order that defines its seed index."""
    specs = [("model.embed_tokens.weight", "q8", (cfg.vocab_size, cfg.dim))]
    for layer in range(cfg.n_layers):
        for suffix, kind, shape in LAYER_TENSORS:
            specs.append((f"model.layers.{layer}.{suffix}", kind, shape(cfg)))
    specs.append(("model.norm.weight", "norm", (cfg.dim,)))
    specs.append(("lm_head.weight", "q8", (cfg.vocab_size, cfg.dim)))
    return specs


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 bit patterns, nearest-even (no NaNs occur in N(0, 0.02) draws)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32)
    bias = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + bias) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def gen_tensor(seed: int, index: int, kind: str, shape: tuple[int, ...]) -> np.ndarray:
    """bf16 bit patterns (uint16) of one tensor."""
    n = int(np.prod(shape))
    if kind == "norm":
        return np.full(n, 0x3F80, dtype=np.uint16)  # 1.0 in bf16
    rng = np.random.Generator(np.random.PCG64([seed, index]))
    return f32_to_bf16_bits(rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))


def seeded_prompt(seed: int, n: int, vocab: int = 32000) -> np.ndarray:
    """n token ids uniform in [3, vocab) -- never the BOS/EOS/unk ids 0..2."""
    rng = np.random.Generator(np.random.PCG64([seed, 0x70726F6D]))
    return rng.integers(3, vocab, size=n, dtype=np.int64).astype(np.int32)


def write_config(path: str, cfg: Config) -> None:
    conf = {
        "architectures": ["LlamaForCausalLM"],
        "model_type": "llama",
        "hidden_size": cfg.dim,
        "intermediate_size": cfg.hidden_dim,
        "num_hidden_layers": cfg.n_layers,
        "num_attention_heads": cfg.n_heads,
        "num_key_value_heads": cfg.n_kv_heads,
        "vocab_size": cfg.vocab_size,
        "max_position_embeddings": cfg.seq_len,
        "rms_norm_eps": 1e-5,
        "rope_theta": 10000.0,
        "torch_dtype": "bfloat16",
    }
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(conf, f, indent=2)


def _safetensors_header(entries: list[tuple[str, tuple[int, ...], int]]) -> bytes:
    """JSON header for bf16 tensors laid out back to back; padded with spaces so that the data
    starts 8-byte aligned and 8 + len(header) is not a multiple of 4096 (the reference parses the
    header straight out of the mmap and relies on a NUL byte after it)."""
    header = {}
    off = 0
    for name, shape, nbytes in entries:
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    raw = json.dumps(header, separators=(",", ":")).encode()
    pad = (-(8 + len(raw))) % 8
    raw += b" " * pad
    if (8 + len(raw)) % 4096 == 0:
        raw += b" " * 8
    return raw


def write_model(path: str, cfg: Config, seed: int, header_only: bool = False) -> list[str]:
    """Write config.json + model.safetensors.  Returns the tensor names in file order."""
    os.makedirs(path, exist_ok=True)
    write_config(path, cfg)
    specs = tensor_specs(cfg)
    entries = [(name, shape, int(np.prod(shape)) * 2) for name, _, shape in specs]
    header = _safetensors_header(entries)
    with open(os.path.join(path, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        if not header_only:
            for idx, (name, kind, shape) in enumerate(specs):
                f.write(gen_tensor(seed, idx, kind, shape).tobytes())
    return [s[0] for s in specs]


def write_q8_cache(cache_dir: str, name: str, q: np.ndarray, s: np.ndarray) -> None:
    """One Q8_0 cache file: int8[n] then fp32[n/32] (src/safetensors.c:110-113)."""
    os.makedirs(cache_dir, exist_ok=True)
    with open(os.path.join(cache_dir, f"{name}-Q8_0.tensor"), "wb") as f:
        f.write(np.ascontiguousarray(q, dtype=np.int8).tobytes())
        f.write(np.ascontiguousarray(s, dtype=np.float32).tobytes())


def write_f32_cache(cache_dir: str, name: str, v: np.ndarray) -> None:
    os.makedirs(cache_dir, exist_ok=True)
    with open(os.path.join(cache_dir, f"{name}-F32.tensor"), "wb") as f:
        f.write(np.ascontiguousarray(v, dtype=np.float32).tobytes())


def write_tokenizer(path: str, vocab_size: int = 32000) -> None:
    """A synthetic tokenizer.bin (src/tokenizer.c:11-48 layout): ints vocab_size,
    max_token_length, bos_id, eos_id; then per piece a float score, an int length and the bytes.
    Pieces: <unk>, <s>, </s>, the 256 byte tokens <0xXX>, " ", then unique letter strings."""
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{i:02X}>" for i in range(256)] + [" "]
    letters = "abcdefghijklmnopqrstuvwxyz"
    seen = set(pieces)
    width = 1
    while len(pieces) < vocab_size:
        for i in range(len(letters) ** width):
            if len(pieces) >= vocab_size:
                break
            s, v = "", i
            for _ in range(width):
                s = letters[v % 26] + s
                v //= 26
            for cand in (s, " " + s):
                if cand not in seen and len(pieces) < vocab_size:
                    pieces.append(cand)
                    seen.add(cand)
        width += 1
    max_len = max(len(p.encode()) for p in pieces)
    with open(path, "wb") as f:
        f.write(struct.pack("<iiii", vocab_size, max_len, 1, 2))
        for i, p in enumerate(pieces):
            b = p.encode()
            score = 0.0 if i < 260 else -float(i)
            f.write(struct.pack("<fi", score, len(b)))
            f.write(b)
