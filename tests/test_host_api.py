"""The reference-compatible host API of libdiolkos.so (include/tensor.h, safetensors.h, sampler.h,
tokenizer.h) on the CPU: the parts that need no GPU -- the tokenizer, the random stream, the
safetensors/JSON loader reading a Q8_0 cache, 16-bit float widening -- against the compiled
reference (oracle/_ref, where it is built) and the Python restatement (oracle/tokenizer_port.py).
"""
import ctypes as C
import json
import os
import shutil
import struct
import subprocess
import sys

import numpy as np
import pytest

from diolkos_b200 import refapi, synth
from oracle import tokenizer_port as TP

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# ---- synthetic tokenizers ----------------------------------------------------------------------
ALPHABET = list("abcdefghij") + ["é", "ß", "日", "本", "😀"]  # 1- to 4-byte code points
NOT_IN_VOCAB = ["z", "ü", "🙂", "\x07"]                         # byte-fallback cases


def write_tokenizer_bin(path, pieces, scores):
    max_len = max(len(p) for p in pieces)
    with open(path, "wb") as f:
        f.write(struct.pack("<iiii", len(pieces), max_len, 1, 2))
        for p, s in zip(pieces, scores):
            f.write(struct.pack("<fi", float(s), len(p)))
            f.write(p)


def make_vocab(seed):
    """<unk>, <s>, </s>, 256 byte pieces, then every substring (and space-prefixed substring) of
    random words; integer scores in [-20, 0] so that equal scores are common (ties between
    candidate merges exercise the leftmost-pair rule)."""
    rng = np.random.default_rng(seed)
    pieces = [b"<unk>", b"<s>", b"</s>"] + [f"<0x{i:02X}>".encode() for i in range(256)]
    seen = set(pieces)
    words = ["".join(rng.choice(ALPHABET, size=rng.integers(2, 8))) for _ in range(60)]
    cands = [" "] + ALPHABET + [" " + a for a in ALPHABET]
    for w in words:
        for i in range(len(w)):
            for j in range(i + 1, len(w) + 1):
                cands += [w[i:j], " " + w[i:j]]
    for c in cands:
        b = c.encode()
        if b not in seen:
            seen.add(b)
            pieces.append(b)
    scores = [0.0] * 259 + [float(rng.integers(-20, 1)) for _ in range(len(pieces) - 259)]
    return pieces, scores, words


def random_texts(seed, words, n=60):
    rng = np.random.default_rng(seed)
    out = [b"", b" ", b"a", "日本".encode(), b"\x80\x80\x80\x80\x80a", b"\xff\xfe", "é😀🙂z".encode()]
    for _ in range(n):
        parts = []
        for _ in range(rng.integers(1, 12)):
            r = rng.random()
            if r < 0.6:
                parts.append(str(rng.choice(words)))
            elif r < 0.8:
                parts.append(str(rng.choice(NOT_IN_VOCAB + ALPHABET)))
            else:
                parts.append(" ")
        out.append("".join(parts).encode())
    return out


@pytest.fixture(scope="module")
def vocab(tmp_path_factory):
    pieces, scores, words = make_vocab(7)
    path = str(tmp_path_factory.mktemp("tok") / "tokenizer.bin")
    write_tokenizer_bin(path, pieces, scores)
    return path, pieces, [np.float32(s) for s in scores], words


def test_encode_matches_port(vocab):
    path, pieces, scores, words = vocab
    tok = refapi.load_tokenizer(path)
    for text in random_texts(1, words):
        for bos, eos in ((True, False), (False, True), (False, False)):
            got = refapi.encode(tok, text, bos, eos)
            want = TP.encode(pieces, scores, text, bos, eos)
            assert got == want, (text, bos, eos)


def test_encode_decode_match_compiled_reference(vocab, ref):
    path, pieces, scores, words = vocab
    R = refapi.bind(ref.lib, names={"build_tokenizer", "encode", "decode", "free_tokenizer"})
    rtok = refapi.load_tokenizer(path, L=R)
    tok = refapi.load_tokenizer(path)
    assert (tok.vocab_size, tok.max_token_length, tok.bos_id, tok.eos_id) == \
        (rtok.vocab_size, rtok.max_token_length, rtok.bos_id, rtok.eos_id)
    for text in random_texts(2, words):
        assert refapi.encode(tok, text) == refapi.encode(rtok, text, L=R), text
    for t in range(len(pieces)):
        for prev in (1, 5):
            assert refapi.decode(tok, prev, t) == refapi.decode(rtok, prev, t, L=R), (prev, t)


def test_encode_long_prompt_matches_port(vocab):
    """A prompt of a few thousand code points (the heap-based merge loop against the rescan)."""
    path, pieces, scores, words = vocab
    rng = np.random.default_rng(3)
    text = " ".join(str(w) for w in rng.choice(words, 400)).encode()
    tok = refapi.load_tokenizer(path)
    assert refapi.encode(tok, text) == TP.encode(pieces, scores, text, True, False)


def test_decode_rules(vocab):
    path, pieces, scores, words = vocab
    tok = refapi.load_tokenizer(path)
    sp = pieces.index(b" a")
    assert refapi.decode(tok, 1, sp) == b"a"           # leading space dropped after BOS
    assert refapi.decode(tok, 7, sp) == b" a"
    assert refapi.decode(tok, 7, 3 + 0x41) == b"A"     # <0x41>
    for t in range(len(pieces)):
        # decode returns a C string: the <0x00> piece reads as empty
        assert refapi.decode(tok, 9, t) == TP.decode(pieces, 9, t).split(b"\0", 1)[0]


def test_safe_printf_filters_control_bytes():
    code = ("from diolkos_b200 import refapi; L = refapi.lib(); "
            "[L.safe_printf(s) for s in (b'ab', b'\\x07', b'\\n', b'', None, b'\\x01x')]; "
            "import ctypes; ctypes.CDLL(None).fflush(None)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, cwd=ROOT, check=True).stdout
    assert out == b"ab\n\x01x"


def test_random_stream(ref):
    L = refapi.lib()
    R = refapi.bind(ref.lib, names={"random_u32", "random_f32"})
    for seed in (1, 42, 0x123456789ABCDEF, 2**63 + 5):
        a, b = C.c_ulonglong(seed), C.c_ulonglong(seed)
        s = seed
        for _ in range(200):
            u = L.random_u32(C.byref(a))
            assert u == R.random_u32(C.byref(b))
            want, s = TP.random_u32(s)
            assert u == want and a.value == s
        f = L.random_f32(C.byref(a))
        assert f == R.random_f32(C.byref(b))
        assert 0.0 <= f < 1.0


def test_half_widening_exact():
    L = refapi.lib()
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([L.f16_to_float(int(v)) for v in h], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(want)])) and np.array_equal(got[np.isinf(want)], want[np.isinf(want)])
    b = np.array([0, 0x3F80, 0xBF80, 0x7F80, 0x0001, 0x8000], np.uint16)
    assert np.array_equal(np.array([L.bf16_to_float(int(v)) for v in b], np.float32), synth.bf16_bits_to_f32(b))


def test_tensor_container():
    L = refapi.lib()
    t = L.tensor_create(64, refapi.Q8_0)
    assert t.contents.dim == 64 and L.Tensor_storage_size(t) == 64 + 2 * 4 and L.tensor_memory(t) == 72
    assert C.addressof(t.contents.scale.contents) == t.contents.data + 64
    assert L.quant_size(refapi.F32) == 4 and L.quant_size(refapi.BF16) == 2 and L.group_size(refapi.Q8_0) == 32
    assert L.convert(t, refapi.Q8_0).contents.data == t.contents.data  # same type: the input itself
    L.tensor_destroy(t)
    assert L.round_down_32(70) == 64 and L.reliable_isnan(float("nan")) and not L.reliable_isnan(1.0)


# ---- loader ------------------------------------------------------------------------------------
SMALL = synth.Config(64, 160, 2, 4, 2, 512, 64)


def _write_small_model(root, name="small-model", seed=5):
    d = os.path.join(root, name)
    synth.write_model(d, SMALL, seed)
    # config.json with the extra members HF configs carry (nested objects, escapes, literals)
    with open(os.path.join(d, "config.json")) as f:
        conf = json.load(f)
    conf.update({"rope_scaling": {"type": "linear", "factor": 2.0, "nested": [1, [2, {"x": None}]]},
                 "name": "café 😀 \"q\" \\ /", "tie_word_embeddings": False, "eps": -1.5e-05})
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(conf, f, indent=1, ensure_ascii=True)
    return d


def _expected_tensors(port, seed=5):
    """name -> ('q8', q, s) or ('f32', v) for the small model."""
    out = {}
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(SMALL)):
        bits = synth.gen_tensor(seed, idx, kind, shape)
        if kind == "q8":
            out[name] = ("q8",) + port.quant_bf16(bits)
        else:
            out[name] = ("f32", synth.bf16_bits_to_f32(bits))
    return out


def _model_tensors(m):
    c = m.config.contents
    got = {"model.embed_tokens.weight": m.token_embedding_table.contents, "model.norm.weight": m.rms_final_weight.contents,
           "lm_head.weight": m.wcls.contents}
    for layer in range(c.n_layers):
        L = m.layers[layer]
        for suffix, field in (("input_layernorm.weight", "rms_att_weight"), ("self_attn.q_proj.weight", "wq"),
                              ("self_attn.k_proj.weight", "wk"), ("self_attn.v_proj.weight", "wv"),
                              ("self_attn.o_proj.weight", "wo"), ("post_attention_layernorm.weight", "rms_ffn_weight"),
                              ("mlp.gate_proj.weight", "w1"), ("mlp.down_proj.weight", "w2"),
                              ("mlp.up_proj.weight", "w3")):
            got[f"model.layers.{layer}.{suffix}"] = getattr(L, field).contents
    return got


def test_loader_reads_the_cache(tmp_path, port, monkeypatch):
    """Q8_0 tensors come from pre-written cache files (no GPU needed); the norms are widened from
    bf16 and their F32 cache files are written like the reference's."""
    d = _write_small_model(str(tmp_path))
    want = _expected_tensors(port)
    cache = os.path.join(str(tmp_path), "cache", "small-model")
    for name, v in want.items():
        if v[0] == "q8":
            synth.write_q8_cache(cache, name, v[1], v[2])
    monkeypatch.chdir(tmp_path)
    m = refapi.lib().load_safetensors(d.encode()).contents
    c = m.config.contents
    assert [c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, c.seq_len] == SMALL.as_list()
    assert m.huggingface_rope
    got = _model_tensors(m)
    assert set(got) == set(want)
    for name, t in got.items():
        if want[name][0] == "q8":
            q, s = t.q8()
            assert np.array_equal(q, want[name][1]) and np.array_equal(s.view(np.uint32), want[name][2].view(np.uint32)), name
        else:
            assert np.array_equal(t.f32(), want[name][1]), name
            with open(os.path.join(cache, f"{name}-F32.tensor"), "rb") as f:
                assert f.read() == want[name][1].tobytes(), name


def test_loader_matches_compiled_reference_cache(tmp_path, ref, monkeypatch):
    """The reference loads the same directory and writes its cache; the library, run where that cache
    is, returns exactly the cached bytes, and writes byte-identical F32 cache files of its own."""
    d = _write_small_model(str(tmp_path))
    work_ref = tmp_path / "ref"
    work_ref.mkdir()
    ref.load(d, str(work_ref))
    ref_cache = work_ref / "cache" / "small-model"
    files = sorted(os.listdir(ref_cache))
    assert len(files) == len(synth.tensor_specs(SMALL))
    mine = tmp_path / "mine"
    (mine / "cache" / "small-model").mkdir(parents=True)
    for f in files:
        if f.endswith("-Q8_0.tensor"):
            shutil.copy(ref_cache / f, mine / "cache" / "small-model" / f)
    monkeypatch.chdir(mine)
    m = refapi.lib().load_safetensors(d.encode()).contents
    for f in files:
        with open(ref_cache / f, "rb") as a, open(mine / "cache" / "small-model" / f, "rb") as b:
            assert a.read() == b.read(), f
    for name, t in _model_tensors(m).items():
        raw = open(ref_cache / f"{name}-{'Q8_0' if t.type == refapi.Q8_0 else 'F32'}.tensor", "rb").read()
        if t.type == refapi.Q8_0:
            q, s = t.q8()
            assert q.tobytes() + s.tobytes() == raw, name
        else:
            assert t.f32().tobytes() == raw, name


def _run_loader(model_dir, cwd):
    code = f"from diolkos_b200 import refapi; refapi.lib().load_safetensors({model_dir!r}.encode())"
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=cwd,
                          env={**os.environ, "PYTHONPATH": ROOT})


def test_loader_missing_tensor_exits(tmp_path, port):
    """A checkpoint without lm_head.weight exits with the reference's message."""
    d = str(tmp_path / "nohead")
    os.makedirs(d)
    synth.write_config(d, SMALL)
    specs = [s for s in synth.tensor_specs(SMALL) if s[0] != "lm_head.weight"]
    entries = [(n, sh, int(np.prod(sh)) * 2) for n, _, sh in specs]
    header = synth._safetensors_header(entries)
    with open(os.path.join(d, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(header)) + header)
        for idx, (name, kind, shape) in enumerate(synth.tensor_specs(SMALL)):
            if name != "lm_head.weight":
                f.write(synth.gen_tensor(5, idx, kind, shape).tobytes())
    # every Q8_0 tensor cached, so that the run needs no GPU before it reaches the check
    want = _expected_tensors(port)
    for name, v in want.items():
        if v[0] == "q8" and name != "lm_head.weight":
            synth.write_q8_cache(str(tmp_path / "cache" / "nohead"), name, v[1], v[2])
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1 and "Missing required tensor: lm_head.weight" in r.stderr, r.stderr


def test_loader_size_mismatch_and_bad_config_exit(tmp_path):
    d = str(tmp_path / "bad")
    synth.write_model(d, SMALL, 5, header_only=True)
    conf = json.load(open(os.path.join(d, "config.json")))
    conf["hidden_size"] = 96
    conf["num_attention_heads"] = 3
    json.dump(conf, open(os.path.join(d, "config.json"), "w"))
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1 and "Tensor size mismatch for model.embed_tokens.weight" in r.stderr, r.stderr
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write('{"hidden_size": 64, "num_hidden_layers": ')
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1 and "config.json" in r.stderr, r.stderr


# ---- corrupt inputs: the loader stops with a message (exit status 1), no GPU needed -------------
def _cached_small_model(tmp_path, port, name="small-model"):
    """The small model with every Q8_0 tensor in the cache (the loader then needs no GPU)."""
    d = _write_small_model(str(tmp_path), name=name)
    cache = os.path.join(str(tmp_path), "cache", name)
    for n, v in _expected_tensors(port).items():
        if v[0] == "q8":
            synth.write_q8_cache(cache, n, v[1], v[2])
    return d, cache


def test_loader_truncated_cache_file_exits(tmp_path, port):
    d, cache = _cached_small_model(tmp_path, port)
    victim = os.path.join(cache, "model.layers.1.mlp.down_proj.weight-Q8_0.tensor")
    size = os.path.getsize(victim)
    with open(victim, "r+b") as f:
        f.truncate(size - 4)  # the last scale cut short
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1 and "is truncated" in r.stderr and "down_proj" in r.stderr, r.stderr


def test_loader_truncated_safetensors_exits(tmp_path, port):
    """A header length past the end of the file: the file is skipped with a message, and the loader
    then stops because the directory holds no usable safetensors file."""
    d, _ = _cached_small_model(tmp_path, port)
    path = os.path.join(d, "model.safetensors")
    with open(path, "rb") as f:
        hlen = struct.unpack("<Q", f.read(8))[0]
    with open(path, "r+b") as f:
        f.truncate(8 + hlen // 2)
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1, r.stderr
    assert "not a safetensors file" in r.stderr and "No safetensors files found" in r.stderr, r.stderr


def test_loader_short_data_section_exits(tmp_path, port):
    """The header is intact but the tensor data stops early: a tensor that is not cached (a norm,
    widened from bf16 on the host) whose bytes lie past the end of the file."""
    d, _ = _cached_small_model(tmp_path, port)
    path = os.path.join(d, "model.safetensors")
    with open(path, "rb") as f:
        hlen = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(hlen))
    ends = {k: v["data_offsets"][1] for k, v in header.items() if k != "__metadata__"}
    norm = max((k for k in ends if k.endswith("layernorm.weight")), key=lambda k: ends[k])
    with open(path, "r+b") as f:
        f.truncate(8 + hlen + ends[norm] - 2)
    r = _run_loader(d, str(tmp_path))
    assert r.returncode == 1 and "Data size mismatch" in r.stderr, r.stderr


def test_tokenizer_truncated_file_exits(tmp_path):
    """tokenizer.bin cut inside a piece, or inside the header: exit status 1 and a message naming the file."""
    pieces, scores, _ = make_vocab(3)
    path = str(tmp_path / "tokenizer.bin")
    write_tokenizer_bin(path, pieces, scores)
    code = f"from diolkos_b200 import refapi; refapi.load_tokenizer({path!r})"
    for cut, what in ((os.path.getsize(path) - 3, "short piece"), (10, "short header")):
        with open(path, "r+b") as f:
            f.truncate(cut)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                           env={**os.environ, "PYTHONPATH": ROOT})
        assert r.returncode == 1 and what in r.stderr and "tokenizer.bin" in r.stderr, r.stderr
