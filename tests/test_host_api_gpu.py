"""The reference-compatible host API (include/transformer.h, safetensors.h, tensor.h, utils.h,
sampler.h) on the GPU: the loader's GPU quantisation and cache files, build_transformer /
forward, sample(), matmul / rmsnorm / softmax, and the localinfer CLI, against the oracle and
(where oracle/_ref is built) the compiled reference."""
import ctypes as C
import os
import struct
import subprocess

import numpy as np
import pytest

from diolkos_b200 import refapi, synth
from oracle import tokenizer_port as TP

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEED = 17


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    root = tmp_path_factory.mktemp("host")
    d = str(root / "tiny-model")
    synth.write_model(d, synth.TINY, SEED)
    return str(root), d


@pytest.fixture(scope="module")
def tiny_weights(port):
    from oracle import load_port_weights

    return load_port_weights(port, synth.TINY, SEED)


@pytest.fixture(scope="module")
def loaded(tiny_dir):
    """load_safetensors with no cache present: every Q8_0 tensor is quantised on the GPU."""
    root, d = tiny_dir
    old = os.getcwd()
    os.chdir(root)
    try:
        m = refapi.lib().load_safetensors(d.encode()).contents
    finally:
        os.chdir(old)
    return m


def _tensors(m):
    from tests.test_host_api import _model_tensors

    return _model_tensors(m)


def test_loader_quantises_like_the_oracle(tiny_dir, loaded, tiny_weights):
    root, d = tiny_dir
    w, by_name = tiny_weights
    cache = os.path.join(root, "cache", "tiny-model")
    for name, t in _tensors(loaded).items():
        want = by_name[name]
        if t.type == refapi.Q8_0:
            q, s = t.q8()
            assert np.array_equal(q, want[0]), name
            assert np.array_equal(s.view(np.uint32), want[1].view(np.uint32)), name
            raw = open(os.path.join(cache, f"{name}-Q8_0.tensor"), "rb").read()
            assert raw == want[0].tobytes() + want[1].tobytes(), name
        else:
            assert np.array_equal(t.f32(), want), name


def test_loader_cache_equals_compiled_reference_cache(tiny_dir, loaded, ref, tmp_path):
    root, d = tiny_dir
    ref.load(d, str(tmp_path))
    mine, theirs = os.path.join(root, "cache", "tiny-model"), tmp_path / "cache" / "tiny-model"
    files = sorted(os.listdir(theirs))
    assert files == sorted(os.listdir(mine))
    for f in files:
        assert open(os.path.join(mine, f), "rb").read() == open(theirs / f, "rb").read(), f


def test_convert_f16_and_f32_match_reference(port, ref):
    """convert() to Q8_0 from F16 and F32 host tensors (GPU quantisers) against the compiled
    reference's convert() on the same tensors, and Q8_0 -> F32 against the oracle's dequantiser."""
    L = refapi.lib()
    R = refapi.bind(ref.lib, names={"convert"})
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(32 * 4096) * 0.05).astype(np.float32)
    x[:32] = 0.0  # an all-zero group
    for qt, arr in ((refapi.F16, x.astype(np.float16)), (refapi.F32, x)):
        arr = np.ascontiguousarray(arr)
        if qt == refapi.F32:
            arr = arr.copy()
            arr[:32] = 1e-3  # the reference's fp32 path divides by a zero scale (NaN); avoid it
        t = refapi.Tensor(type=qt, data=arr.ctypes.data, dim=arr.size, hdim=arr.size, vdim=1)
        got = L.convert(C.byref(t), refapi.Q8_0).contents
        want = R.convert(C.byref(t), refapi.Q8_0).contents
        gq, gs = got.q8()
        wq, ws = want.q8()
        assert np.array_equal(gq, wq), qt
        assert np.array_equal(np.nan_to_num(gs), np.nan_to_num(ws)), qt
    back = L.convert(C.byref(got), refapi.F32).contents.f32()
    np.testing.assert_array_equal(back, port.dequant(gq, gs))


@pytest.fixture(scope="module")
def transformer(tiny_dir, loaded):
    root, d = tiny_dir
    t = refapi.Transformer()
    old = os.getcwd()
    os.chdir(root)
    try:
        refapi.lib().build_transformer_from_safetensors(C.byref(t), d.encode())
    finally:
        os.chdir(old)
    yield t
    refapi.lib().free_transformer(C.byref(t))


def test_forward_matches_oracle(transformer, port, tiny_weights):
    """The reference-API forward() against the oracle at the first positions (no int8 flip can occur
    yet), and bit-identical to the engine's own step (dk_model_forward) at every position: the engine's
    per-layer parity with the reference is gated in test_model_gpu.py."""
    from diolkos_b200.model import Model
    from oracle import PortModel

    w, by_name = tiny_weights
    cfg = synth.TINY
    c = transformer.config
    assert [c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, c.seq_len] == cfg.as_list()
    pm = PortModel(port, cfg, w)
    eng = Model(cfg)
    eng.load_named(by_name)
    eng.finalize()
    L = refapi.lib()
    seq = list(synth.seeded_prompt(23, 12))
    errs = []
    for pos, tok in enumerate(seq):
        lt = L.forward(C.byref(transformer), int(tok), pos)
        assert C.addressof(lt.contents) == C.addressof(transformer.state.logits.contents)
        a = lt.contents.f32()
        np.testing.assert_array_equal(a, eng.forward(int(tok), pos), err_msg=f"position {pos}")
        if pos < 3:
            b = pm.forward(int(tok), pos)
            errs.append(np.max(np.abs(a - b)) / np.max(np.abs(b)))
    eng.close()
    assert max(errs) < 1e-5, errs


def _probs(logits, temperature):
    z = (logits / np.float32(temperature)).astype(np.float64)
    e = np.exp(z - z.max())
    return e / e.sum()


@pytest.mark.parametrize("temperature,topp", [(0.0, 0.9), (1.0, 0.0), (0.7, 1.0), (0.8, 0.9), (1.2, 0.5)])
def test_sample_matches_reference_sampler(port, temperature, topp):
    """sample() (dk_sample on the GPU, coin from the host xorshift stream) against the oracle
    sampler: the same random stream, the same token except where the coin falls within float
    rounding of a cumulative-probability boundary, and the probabilities written back into the
    logits like the reference."""
    L = refapi.lib()
    rng = np.random.default_rng(int(temperature * 10 + topp * 100))
    V = 32000
    s = refapi.Sampler()
    L.build_sampler(C.byref(s), V, temperature, topp, 1234)
    state = 1234
    mism = 0
    for it in range(72):
        heavy = it % 6 == 5  # few distinct values: tie groups of thousands of tokens
        if heavy:
            logits = np.round(rng.standard_normal(V) * 2).astype(np.float32)
        else:
            logits = (rng.standard_normal(V) * (1 + it % 5)).astype(np.float32)
        if it % 7 == 0:
            logits[rng.integers(0, V, 5)] = logits.max()  # a small tie group at the top
        buf = logits.copy()
        coin = TP.random_f32(state)[0] if temperature > 0 else None
        tok = L.sample(C.byref(s), buf.ctypes.data_as(C.POINTER(C.c_float)))
        want, state = port.sample(logits, temperature, topp, state)
        assert s.rng_state == state
        if temperature == 0.0:
            assert tok == want == int(np.argmax(logits))
            np.testing.assert_array_equal(buf, logits)
            continue
        p = _probs(logits, temperature)
        np.testing.assert_allclose(buf, p, rtol=2e-5, atol=1e-9)
        if tok == want:
            continue
        if heavy and abs(tok - want) <= 64 and (buf[tok] == buf[want] or not 0 < topp < 1):
            # thousands of equal small probabilities: the reference's float32 running sum drifts by
            # ~1e-4 over the vocabulary, a few elements' worth, from the exact (or tree-summed)
            # cumulative; top-p picks inside a tie group from the group's start sum
            continue
        # otherwise only a coin within float rounding of a cumulative-probability boundary (or a
        # cumulative sum within rounding of topp) may pick the neighbouring token
        mism += 1
        if 0 < topp < 1:
            kept = np.sort(p[p >= (1 - topp) / (V - 1)])[::-1]
            cum = np.cumsum(kept)
            last = int(np.argmax(cum > topp)) if (cum > topp).any() else len(cum) - 1
            near = min(np.min(np.abs(cum - coin * cum[last])), np.min(np.abs(cum - topp)))
        else:
            near = np.min(np.abs(np.cumsum(p) - coin))
        assert near < (1e-4 if heavy else 1e-5), (it, tok, want, near)
    assert mism <= 3
    L.free_sampler(C.byref(s))


def test_utils_on_host_tensors(port):
    L = refapi.lib()
    rng = np.random.default_rng(8)
    n, d = 4096, 1000
    wq = rng.integers(-127, 128, n * d).astype(np.int8)
    ws = (rng.random(n * d // 32) * 0.01 + 1e-4).astype(np.float32)
    W = L.tensor_create(n * d, refapi.Q8_0)
    C.memmove(W.contents.data, wq.ctypes.data, wq.nbytes)
    C.memmove(W.contents.scale, ws.ctypes.data, ws.nbytes)
    x = rng.standard_normal(n).astype(np.float32)
    X = L.tensor_create(n, refapi.F32)
    C.memmove(X.contents.data, x.ctypes.data, x.nbytes)
    O = L.tensor_create(d, refapi.F32)
    for _ in range(2):  # the second call uses the packed copy kept from the first
        L.matmul(O, X, W, n, d)
        np.testing.assert_array_equal(O.contents.f32(), port.matmul(x, wq, ws, n, d))
    w = rng.random(n).astype(np.float32)
    Wn = L.tensor_create(n, refapi.F32)
    C.memmove(Wn.contents.data, w.ctypes.data, w.nbytes)
    O2 = L.tensor_create(n, refapi.F32)
    L.rmsnorm(O2, X, Wn, n)
    np.testing.assert_allclose(O2.contents.f32(), port.rmsnorm(x, w), rtol=2e-6, atol=1e-7)
    L.softmax(X, n)
    np.testing.assert_allclose(X.contents.f32(), port.softmax(x), rtol=2e-6, atol=1e-12)
    for t in (W, X, O, Wn, O2):
        L.tensor_destroy(t)


def test_localinfer_greedy(tiny_dir, loaded, tiny_weights, tmp_path):
    """bin/localinfer -t 0 prints the pieces of the engine's greedy continuation of the encoded
    prompt, stopping like the reference's generate()."""
    from diolkos_b200.model import Model

    root, d = tiny_dir
    tok_path = str(tmp_path / "tokenizer.bin")
    synth.write_tokenizer(tok_path, synth.TINY.vocab_size)
    pieces, scores, *_ = TP.load(tok_path)
    prompt = b"abc de fgh"
    steps = 48
    ids = TP.encode(pieces, scores, prompt, True, False)
    w, by_name = tiny_weights
    m = Model(synth.TINY)
    m.load_named(by_name)
    m.finalize()
    gen = [int(t) for t in m.generate(np.array(ids, np.int32), steps)]
    m.close()
    seq = ids[: min(len(ids), steps)] + gen
    text = b""
    for pos in range(1, min(len(seq), steps + 1)):
        nxt = seq[pos]
        if nxt == 1:
            break
        piece = TP.decode(pieces, seq[pos - 1], nxt).split(b"\0", 1)[0]
        if len(piece) == 1 and not (32 <= piece[0] < 127 or piece[0] in b" \t\n\v\f\r"):
            continue
        text += piece
    exe = os.path.join(ROOT, "diolkos_b200", "bin", "localinfer")
    r = subprocess.run([exe, d, "-t", "0", "-n", str(steps), "-i", prompt.decode(), "-z", tok_path],
                       capture_output=True, cwd=root, timeout=300)
    assert r.returncode == 0, r.stderr.decode()
    out = r.stdout.split(b"Loaded ")[1].split(b"\n", 1)[1]
    assert out == text + b"\n", (out[:200], text[:200])
    assert b"achieved tok/s" in r.stderr
    # The reference's own, unmodified src/bin/localinfer.c (+ transformer_info.c), compiled against
    # include/ and linked with libdiolkos.so (oracle Makefile, target dropin), prints the same text.
    dropin = os.path.join(ROOT, "oracle", "_ref", "dropin", "localinfer")
    if not os.path.exists(dropin):
        pytest.skip("oracle/_ref/dropin/localinfer not built here")
    r2 = subprocess.run([dropin, d, "-t", "0", "-n", str(steps), "-i", prompt.decode(), "-z", tok_path],
                        capture_output=True, cwd=root, timeout=300)
    assert r2.returncode == 0, r2.stderr.decode()
    assert r2.stdout.endswith(text + b"\n"), r2.stdout[-300:]
    assert b"achieved tok/s" in r2.stderr


def _run_cli(exe, model_dir, tok_path, prompt, steps, cwd, extra=()):
    r = subprocess.run([exe, model_dir, "-t", "0", "-n", str(steps), "-i", prompt, "-z", tok_path, *extra],
                       capture_output=True, cwd=cwd, timeout=300)
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return r


def test_client_cli_one_gpu(tiny_dir, loaded, tmp_path):
    """bin/client (the reference client's flags, ranks = GPUs of this box) with one rank prints what
    bin/localinfer prints."""
    root, d = tiny_dir
    tok_path = str(tmp_path / "tokenizer.bin")
    synth.write_tokenizer(tok_path, synth.TINY.vocab_size)
    bin_dir = os.path.join(ROOT, "diolkos_b200", "bin")
    a = _run_cli(os.path.join(bin_dir, "localinfer"), d, tok_path, "abc de fgh", 40, root)
    b = _run_cli(os.path.join(bin_dir, "client"), d, tok_path, "abc de fgh", 40, root, ("-g", "1"))
    text = a.stdout.split(b"Loaded ")[1].split(b"\n", 1)[1]
    assert b.stdout.endswith(text), (b.stdout[-200:], text[-200:])
    assert b"achieved tok/s" in b.stderr


def _gpus() -> int:
    import torch

    return torch.cuda.device_count()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_client_cli_two_gpus(loaded, tmp_path):
    """Two ranks (one process per GPU, the sums exchanged over NVLink) run the same generate loop; the
    tensor-parallel sum order moves logits by ~1e-6 relative, so the greedy text agrees with one GPU's
    except after a near-tie: the first pieces are compared.  The model is a small one that splits over
    two ranks (4 heads of 64 dims, hidden 768: 128 dims and 384 hidden rows per rank; the tiny model's
    6 heads of 48 do not split into 32-multiples)."""
    cfg = synth.TINY.replace(dim=256, n_heads=4, n_kv_heads=4)
    d = str(tmp_path / "tp-model")
    synth.write_model(d, cfg, SEED)
    tok_path = str(tmp_path / "tokenizer.bin")
    synth.write_tokenizer(tok_path, cfg.vocab_size)
    exe = os.path.join(ROOT, "diolkos_b200", "bin", "client")
    prompt = b"abc de fgh"
    one = _run_cli(exe, d, tok_path, prompt.decode(), 24, str(tmp_path), ("-g", "1"))
    two = _run_cli(exe, d, tok_path, prompt.decode(), 24, str(tmp_path), ("-g", "2"))
    assert b"(2 GPUs)" in two.stderr

    def generated(out: bytes) -> bytes:  # rank 0 echoes the prompt, then prints the pieces; other ranks
        i = out.find(prompt)              # may print their loading lines anywhere around it
        assert i >= 0, out[-300:]
        return out[i + len(prompt):].split(b"\n", 1)[0]

    g1, g2 = generated(one.stdout), generated(two.stdout)
    first = g1.split(b" ", 1)[0]  # the first generated piece(s) before a space
    assert len(g2) > 0 and len(first) > 0 and g2.startswith(first), (g1[:80], g2[:80])
