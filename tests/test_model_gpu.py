"""The whole decode step on the GPU (dk_model_*: one CUDA graph per token) against the reference.

Parity is measured checkpoint by checkpoint with tests/parity.py: the hooked reference build (the
reference's unmodified forward() with its rmsnorm / matmul inputs recorded) where the reference has the
configuration (bf16 KV cache), the restatement (oracle/port.c, pinned to the reference) for fp32 KV
caches.  Every position is run state-synchronised (the oracle's KV history written into the GPU cache
first), and the tests assert, at every position:
  * every GEMV + residual add of the GPU step is bit-exact, replayed from the GPU's own activations;
  * every int8 activation that differs from the oracle's is a +-1 flip at a value that lies between the
    rounding boundary and the GPU's own value (the reference's libmvec expf and AVX2 sum order cannot
    be reproduced bit for bit, so fp32 inputs of a quantisation can differ by a few ulp);
  * before a step's first flip, every checkpoint -- the residual stream after each residual add, the
    attention and SwiGLU outputs, the logits -- agrees within 1e-3 relative.
Free-running greedy generation is compared token by token with the reference's own greedy stream: the
number of identical tokens is reported, and a divergence before token 64 must sit at a near-tie that the
measured logit difference covers."""
import os

import numpy as np
import pytest

from diolkos_b200 import synth
from tests import parity
from tests.golden import make_golden as G

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _first_div(a, b):
    m = min(len(a), len(b))
    for i in range(m):
        if a[i] != b[i]:
            return i
    return m


@pytest.fixture(scope="module")
def tiny_weights(port):
    from oracle import load_port_weights

    return load_port_weights(port, synth.TINY, G.TINY_SEED)


def _gpu_model(cfg, by_name, kv_f32=False):
    from diolkos_b200.model import Model

    m = Model(cfg, kv_f32=kv_f32)
    m.load_named(by_name)
    m.finalize()
    return m


def _norms(w, cfg):
    """The norm weights of the GEMV ops that carry an rmsnorm prologue, per op (None for the others)."""
    from oracle import PW_RMS_ATT, PW_RMS_FFN, PW_RMS_FINAL

    out = []
    for l in range(cfg.n_layers):
        out += [np.asarray(w[(PW_RMS_ATT, l)], np.float32), None, np.asarray(w[(PW_RMS_FFN, l)], np.float32), None]
    return out + [np.asarray(w[(PW_RMS_FINAL, -1)], np.float32)]


def _hooked_ref():
    from oracle import Ref, ref_path

    if ref_path("portable", hooked=True) is None:
        pytest.skip("the hooked reference build (oracle/_ref) is not present")
    return Ref("portable", hooked=True)


def _check(recs, label):
    """The harness's assertions over a synchronised run (tests/parity.py: check)."""
    print(parity.check(recs, label))


def test_tiny_logits_match_reference_golden(tiny_weights):
    """The first positions against the reference's committed golden logits (no flip possible yet)."""
    w, by_name = tiny_weights
    tg = np.load(os.path.join(GOLD, "tiny.npz"))
    ps = G.TINY_PROMPTS[0]
    prompt = synth.seeded_prompt(ps, 8)
    m = _gpu_model(synth.TINY, by_name)
    for pos in range(3):
        lg = m.forward(int(prompt[pos]), pos)
        gl = tg[f"logits_{ps}_{pos}"]
        assert parity.rel(lg, gl) < 1e-5, pos


def test_tiny_per_layer_parity_vs_reference(tiny_weights, port):
    """Config 1 (tiny model, bf16 KV, 8-token prompts), every position of the reference's own greedy
    continuation (136 positions per prompt, 3 prompts), state-synchronised against the hooked reference:
    per-layer checkpoints within 1e-3 before each step's first flip, every flip attributed, every GEMV
    replay bit-exact."""
    w, by_name = tiny_weights
    cfg = synth.TINY
    ref = _hooked_ref()
    tg = np.load(os.path.join(GOLD, "tiny.npz"))
    tmp = __import__("tempfile").mkdtemp()
    md = os.path.join(tmp, "tiny")
    synth.write_model(md, cfg, G.TINY_SEED)
    for ps in G.TINY_PROMPTS:
        prompt = synth.seeded_prompt(ps, 8)
        seq = list(prompt) + list(tg[f"tokens_{ps}"])
        gpu = _gpu_model(cfg, by_name)
        gpu.dump_enable()
        recs = parity.synced_run(gpu, ref.load(md, tmp), seq, min(len(seq), G.TINY_STEPS), port, w, _norms(w, cfg),
                                 cfg)
        _check(recs, f"tiny prompt {ps}")
        # the reference's greedy token wherever no flip touched the step and the top-2 gap is not a tie
        for r in recs:
            if not r["n_flips"] and r["top2_gap"] > 10 * r["logits_rel"]:
                assert r["argmax"][0] == r["argmax"][1], (ps, r["pos"])


def test_tiny_greedy_tokens_vs_reference(tiny_weights):
    """The north-star gate on config 1: free-running greedy generation (the whole loop on the GPU) against
    the reference's own greedy tokens (golden), 128 tokens per prompt.  The count of identical tokens is
    reported per prompt.  Where a prompt diverges before token 64, the divergence must be a near-tie:
    the reference's logit margin between its token and the GPU's token is within the measured
    GPU-vs-reference logit difference at that position, the histories being identical up to there."""
    w, by_name = tiny_weights
    tg = np.load(os.path.join(GOLD, "tiny.npz"))
    cfg = synth.TINY
    ref = _hooked_ref()
    tmp = __import__("tempfile").mkdtemp()
    md = os.path.join(tmp, "tiny")
    synth.write_model(md, cfg, G.TINY_SEED)
    counts = {}
    for ps in G.TINY_PROMPTS:
        prompt = synth.seeded_prompt(ps, 8)
        m = _gpu_model(cfg, by_name)
        gpu = m.generate(prompt, G.TINY_STEPS)
        rtok = tg[f"tokens_{ps}"]
        n = _first_div(gpu, rtok)
        counts[ps] = n
        if n >= min(64, len(rtok)):
            continue
        # teacher-forced (not synchronised) up to the divergence: the same tokens on both sides
        seq = list(prompt) + list(rtok)
        rm, gm = ref.load(md, tmp), _gpu_model(cfg, by_name)
        p_div = len(prompt) - 1 + n
        for pos in range(p_div + 1):
            lo = rm.forward(int(seq[pos]), pos)
            lg = gm.forward(int(seq[pos]), pos)
        a_ref, a_gpu = int(np.argmax(lo)), int(np.argmax(lg))
        assert a_ref == int(rtok[n]) and a_gpu == int(gpu[n]), (ps, n)
        margin = float(lo[a_ref] - lo[a_gpu])
        diff = float(np.max(np.abs(lg - lo)))
        assert margin <= 2.0 * diff, (ps, n, margin, diff)
    print("identical greedy tokens (of 128) per prompt:", counts)


def test_tiny_synced_vs_oracle_random_tokens(port, tiny_weights):
    """Random tokens (not the reference's stream), 48 positions, state-synchronised against the
    restatement with the same bf16 cache."""
    from oracle import PortModel

    w, by_name = tiny_weights
    cfg = synth.TINY
    gpu = _gpu_model(cfg, by_name)
    gpu.dump_enable()
    pm = PortModel(port, cfg, w)
    seq = list(synth.seeded_prompt(11, 8)) + list(np.random.default_rng(0).integers(3, cfg.vocab_size, 40))
    _check(parity.synced_run(gpu, pm, seq, len(seq), port, w, _norms(w, cfg), cfg), "tiny random tokens")


def test_generate_equals_forward_argmax(tiny_weights):
    """The on-device greedy loop and the host loop over forward() produce the same tokens."""
    w, by_name = tiny_weights
    cfg = synth.TINY
    m = _gpu_model(cfg, by_name)
    prompt = synth.seeded_prompt(9, 8)
    gen = m.generate(prompt, 40)
    m2 = _gpu_model(cfg, by_name)
    tok, out = int(prompt[0]), []
    for pos in range(40):
        lg = m2.forward(tok, pos)
        nxt = int(prompt[pos + 1]) if pos < len(prompt) - 1 else int(np.argmax(lg))
        if pos >= len(prompt) - 1:
            out.append(nxt)
        if nxt == 1:
            break
        tok = nxt
    np.testing.assert_array_equal(gen, np.array(out, np.int32))


@pytest.mark.parametrize("wide_from", [None, 100])
def test_kv_f32_and_gqa_vs_oracle(port, wide_from, monkeypatch):
    """fp32 KV cache and grouped-query attention (8 query heads per KV head, as in 70B), against the
    restatement with the same cache type, state-synchronised over 300 positions (several attention
    splits); with wide_from = 100 the attention takes its wide form (CTA-wide items) from position 100."""
    from oracle import PortModel, load_port_weights

    if wide_from is not None:
        monkeypatch.setenv("DIOLKOS_ATTN_WIDE_FROM", str(wide_from))
    cfg = synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=1, vocab_size=2048, seq_len=512)
    w, by_name = load_port_weights(port, cfg, 77)
    for kv_f32 in (True, False):
        m = _gpu_model(cfg, by_name, kv_f32=kv_f32)
        m.dump_enable()
        pm = PortModel(port, cfg, w, kv_f32=kv_f32)
        seq = np.random.default_rng(1).integers(3, cfg.vocab_size, 300)
        _check(parity.synced_run(m, pm, seq, len(seq), port, w, _norms(w, cfg), cfg), f"gqa kv_f32={kv_f32}")


def test_device_weight_upload_path(torch_cuda_fixture=None):
    """Weights quantised on the GPU and set from device memory give the same model as the host
    path (quantised by the oracle, which is bit-exact with the reference's loader)."""
    import torch

    from diolkos_b200 import ops
    from diolkos_b200.model import Model, weight_id
    from oracle import Port, load_port_weights

    cfg = synth.Config(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=4, vocab_size=1024, seq_len=64)
    port = Port()
    _, by_name = load_port_weights(port, cfg, 5)
    host = Model(cfg)
    host.load_named(by_name)
    host.finalize()
    dev = Model(cfg)
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        bits = synth.gen_tensor(5, idx, kind, shape)
        which, layer = weight_id(name)
        if kind == "q8":
            q, s = ops.quantize_bf16(torch.from_numpy(bits.view(np.int16)).cuda())
            torch.cuda.synchronize()
            dev.set_weight_device(which, layer, q, s)
        else:
            dev.set_weight_device(which, layer, torch.from_numpy(synth.bf16_bits_to_f32(bits)).cuda())
    dev.finalize()
    for pos, tok in enumerate([5, 17, 900, 3]):
        np.testing.assert_array_equal(host.forward(tok, pos), dev.forward(tok, pos))


def test_bad_arguments_fail_loudly():
    from diolkos_b200._native import DiolkosError
    from diolkos_b200.model import Model

    with pytest.raises(DiolkosError):
        Model(synth.Config(dim=100, hidden_dim=64, n_layers=1, n_heads=3, n_kv_heads=3, vocab_size=10, seq_len=8))
    m = Model(synth.Config(dim=64, hidden_dim=64, n_layers=1, n_heads=2, n_kv_heads=2, vocab_size=64, seq_len=8))
    with pytest.raises(DiolkosError):
        m.finalize()  # weights missing
    with pytest.raises(DiolkosError):
        m.forward(0, 0)  # not finalized


def test_dim4096_model_vs_oracle(port):
    """dim 4096 on 256 threads takes the one-round-trip rmsnorm prologue (its own sum order):
    state-synchronised against the restatement, fp32 KV."""
    from oracle import PortModel, load_port_weights

    cfg = synth.Config(dim=4096, hidden_dim=1024, n_layers=1, n_heads=32, n_kv_heads=8, vocab_size=1000, seq_len=64)
    w, by_name = load_port_weights(port, cfg, 91)
    m = _gpu_model(cfg, by_name, kv_f32=True)
    m.dump_enable()
    pm = PortModel(port, cfg, w, kv_f32=True)
    seq = np.random.default_rng(2).integers(3, cfg.vocab_size, 24)
    _check(parity.synced_run(m, pm, seq, len(seq), port, w, _norms(w, cfg), cfg), "dim4096")


# 32 KV heads of 32 dims: the decode attention's split count reaches its cap (ceil(5 * SMs / 32): 24 on
# 148 SMs) at position 384, where a chunk rounded up can leave the last split without positions.
CAPPED = synth.Config(dim=1024, hidden_dim=256, n_layers=2, n_heads=32, n_kv_heads=32, vocab_size=256, seq_len=600)


def test_capped_split_plan_vs_oracle(port):
    """Decode through the positions where the split count is capped (385 .. 529 had an empty last split
    under a plan that fixed the count before the chunk): state-synchronised against the restatement at
    every position up to 560, finite logits from 370 on."""
    from oracle import PortModel, load_port_weights

    w, by_name = load_port_weights(port, CAPPED, 93)
    m = _gpu_model(CAPPED, by_name, kv_f32=True)
    m.dump_enable()
    pm = PortModel(port, CAPPED, w, kv_f32=True)
    seq = np.random.default_rng(3).integers(3, CAPPED.vocab_size, 560)
    recs = parity.synced_run(m, pm, seq, len(seq), port, w, _norms(w, CAPPED), CAPPED)
    _check(recs, "capped split plan")


def _logits_bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize(
    "shape,kv_f32,P,wide_from",
    [
        ("tiny", False, 8, None),
        ("tiny", False, 200, None),
        ("tiny", True, 200, 0),      # the wide attention form at every position
        ("gqa", True, 300, None),    # two prefill chunks (256 + 43 positions), many attention splits
        ("gqa", False, 300, None),
        ("gqa", True, 300, 0),       # wide items over 8 query heads, 80-position splits
        ("gqa", False, 300, 100),    # the form switches inside the first chunk
        ("wide", True, 40, None),    # dim 4096: the one-round-trip rmsnorm prologue
        ("capped", False, 540, 384),   # 32 KV heads: the narrow split count is capped (23 on 148 SMs) from
                                       # position 369; the wide form takes over at 384
        ("capped", True, 540, None),   # the default: on 148 SMs the narrow form throughout (4 x 32 wide
                                       # items would leave 20 CTAs idle)
        ("swiglu", True, 100, None),   # hidden 4096: w1|w3 (8192 rows) on the pipelined tensor-core matmul
    ],
)
def test_prefill_equals_decode_steps(port, tiny_weights, shape, kv_f32, P, wide_from, monkeypatch):
    """The batched prefill (tensor-core matmuls over the prompt positions) leaves the KV cache exactly
    as decode steps at those positions do (every model here has 2 layers or more: the prefill stops
    after the last layer's K/V rows, so only earlier layers run attention and the MLP): the logits of the
    last prompt position, decoded after the prefill, equal bit for bit those decoded after stepping every
    prompt position.  wide_from moves the position from which the attention runs in its wide form
    (DIOLKOS_ATTN_WIDE_FROM; None: the default, 384)."""
    from oracle import load_port_weights

    if wide_from is not None:
        monkeypatch.setenv("DIOLKOS_ATTN_WIDE_FROM", str(wide_from))

    if shape == "tiny":
        cfg, by_name = synth.TINY, tiny_weights[1]
    elif shape == "gqa":
        cfg = synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=1, vocab_size=2048, seq_len=512)
        by_name = load_port_weights(port, cfg, 77)[1]
    elif shape == "swiglu":
        cfg = synth.Config(dim=512, hidden_dim=4096, n_layers=2, n_heads=8, n_kv_heads=8, vocab_size=512, seq_len=128)
        by_name = load_port_weights(port, cfg, 95)[1]
    elif shape == "capped":
        cfg, by_name = CAPPED, load_port_weights(port, CAPPED, 93)[1]
    else:
        cfg = synth.Config(dim=4096, hidden_dim=1024, n_layers=2, n_heads=32, n_kv_heads=8, vocab_size=1000, seq_len=64)
        by_name = load_port_weights(port, cfg, 91)[1]
    m = _gpu_model(cfg, by_name, kv_f32=kv_f32)
    prompt = np.random.default_rng(P).integers(3, cfg.vocab_size, P).astype(np.int32)
    m.set_tokens(prompt, n_forced=P)
    m.prefill(0, P - 1)
    after_prefill = m.forward(int(prompt[P - 1]), P - 1)
    for pos in range(P):  # the same positions as decode steps (they overwrite the cache entries)
        stepped = m.forward(int(prompt[pos]), pos)
    np.testing.assert_array_equal(_logits_bits(after_prefill), _logits_bits(stepped))


def test_generate_with_prefill_equals_stepped_prompt(tiny_weights):
    """dk_model_generate prefills the forced prompt positions; the generated tokens equal those of
    the loop that steps every prompt position (DIOLKOS_PREFILL=0)."""
    cfg, by_name = synth.TINY, tiny_weights[1]
    m = _gpu_model(cfg, by_name)
    prompt = synth.seeded_prompt(5, 40)
    gen = m.generate(prompt, 120)
    os.environ["DIOLKOS_PREFILL"] = "0"
    try:
        stepped = m.generate(prompt, 120)
    finally:
        del os.environ["DIOLKOS_PREFILL"]
    assert len(gen) > 0
    np.testing.assert_array_equal(gen, stepped)


def _device_model(cfg, seed, kv_f32=True):
    """A seeded random model built on the GPU (bf16 N(0, 0.02) weights quantised by the library)."""
    import torch

    from diolkos_b200 import ops
    from diolkos_b200.model import Model, weight_id

    m = Model(cfg, kv_f32=kv_f32)
    g = torch.Generator(device="cuda")
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        which, layer = weight_id(name)
        n = int(np.prod(shape))
        if kind == "norm":
            m.set_weight_device(which, layer, torch.ones(n, device="cuda", dtype=torch.float32))
            continue
        g.manual_seed(seed * 1000003 + idx)
        w = (torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)
        q, s = ops.quantize_bf16(w.view(torch.int16))
        m.set_weight_device(which, layer, q, s)
    m.finalize()
    return m


def test_70b_shape_layer_prefill_and_decode():
    """Two layers of the 70B shape (dim 8192, hidden 28672, 64 heads over 8 KV heads): the wide
    activation prologue, 28672-column matmuls on the tensor cores and 8 query heads per KV head in the
    prefill attention.  The prefill leaves the KV cache stepped decode leaves (bit-exact logits
    after it), logits are finite, and generate equals the argmax over forward."""
    cfg = synth.LLAMA70B.replace(n_layers=2, seq_len=256)
    m = _device_model(cfg, 70)
    P = 150
    prompt = np.random.default_rng(70).integers(3, cfg.vocab_size, P).astype(np.int32)
    m.set_tokens(prompt, n_forced=P)
    m.prefill(0, P - 1)
    after_prefill = m.forward(int(prompt[P - 1]), P - 1)
    assert np.isfinite(after_prefill).all()
    for pos in range(P):
        stepped = m.forward(int(prompt[pos]), pos)
    np.testing.assert_array_equal(_logits_bits(after_prefill), _logits_bits(stepped))
    gen = m.generate(prompt[:8], 24)
    tok, out = int(prompt[0]), []
    for pos in range(24):
        lg = m.forward(tok, pos)
        nxt = int(prompt[pos + 1]) if pos < 7 else int(np.argmax(lg))
        if pos >= 7:
            out.append(nxt)
        if nxt == 1:
            break
        tok = nxt
    np.testing.assert_array_equal(gen, np.array(out, np.int32))


def _gpu_generated_weights(cfg, seed):
    """A seeded model generated on the GPU (bf16 N(0, 0.02), quantised by the library's quantiser, which
    is bit-exact with the reference's loader) and brought to the host: {HF name: (q, s) or fp32 vector}
    and the restatement's weight dict."""
    import torch

    from diolkos_b200 import ops
    from diolkos_b200.model import weight_id

    by_name, w = {}, {}
    g = torch.Generator(device="cuda")
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        n = int(np.prod(shape))
        if kind == "norm":
            val = np.ones(n, np.float32)
        else:
            g.manual_seed(seed * 1000003 + idx)
            x = (torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)
            q, s_ = ops.quantize_bf16(x.view(torch.int16))
            torch.cuda.synchronize()
            val = (q.cpu().numpy(), s_.cpu().numpy())
        by_name[name] = val
        which, layer = weight_id(name)
        w[(_PORT_KEY[which], layer)] = val
    return by_name, w


def _port_key_map():
    import oracle
    from diolkos_b200 import _native as N

    return {N.DK_W_EMB: oracle.PW_EMB, N.DK_W_RMS_FINAL: oracle.PW_RMS_FINAL, N.DK_W_WCLS: oracle.PW_WCLS,
            N.DK_W_RMS_ATT: oracle.PW_RMS_ATT, N.DK_W_WQ: oracle.PW_WQ, N.DK_W_WK: oracle.PW_WK,
            N.DK_W_WV: oracle.PW_WV, N.DK_W_WO: oracle.PW_WO, N.DK_W_RMS_FFN: oracle.PW_RMS_FFN,
            N.DK_W_W1: oracle.PW_W1, N.DK_W_W2: oracle.PW_W2, N.DK_W_W3: oracle.PW_W3}


_PORT_KEY = _port_key_map()


def _write_ref_cache(tmp, name, cfg, by_name):
    """The model for the reference loader: config.json + header-only safetensors + the Q8_0 / F32 cache
    files it reads instead of quantising (src/safetensors.c:57-114)."""
    md = os.path.join(tmp, name)
    synth.write_model(md, cfg, 0, header_only=True)
    cache = os.path.join(tmp, "cache", name)
    for tname, kind, _ in synth.tensor_specs(cfg):
        v = by_name[tname]
        if kind == "q8":
            synth.write_q8_cache(cache, tname, v[0], v[1])
        else:
            synth.write_f32_cache(cache, tname, v)
    return md


def test_llama7b_shape_layers_vs_reference(port):
    """The 7B shape itself (dim 4096, hidden 11008, 32 heads, vocab 32000) with 2 layers, bf16 KV, against
    the hooked reference, state-synchronised over a seeded 48-token sequence: per-layer checkpoints within
    1e-3 before each step's first flip, every flip attributed, every GEMV replay bit-exact."""
    import tempfile

    from diolkos_b200.model import Model

    ref = _hooked_ref()
    cfg = synth.LLAMA7B.replace(n_layers=2, seq_len=128)
    by_name, w = _gpu_generated_weights(cfg, 7)
    tmp = tempfile.mkdtemp()
    md = _write_ref_cache(tmp, "llama7b_l2", cfg, by_name)
    gpu = Model(cfg)
    gpu.load_named(by_name)
    gpu.finalize()
    gpu.dump_enable()
    seq = synth.seeded_prompt(7, 48, cfg.vocab_size)
    recs = parity.synced_run(gpu, ref.load(md, tmp), seq, len(seq), port, w, _norms(w, cfg), cfg)
    _check(recs, "llama2-7b shape, 2 layers")
