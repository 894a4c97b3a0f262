"""The whole decode step on the GPU (dk_model_*: one CUDA graph per token) vs the oracle and the
reference's golden outputs.

Tolerances.  The reference re-quantises its fp32 activations to int8 before every matmul, so an
ulp-level difference anywhere upstream (its vectorised expf and rsqrt approximation cannot be
reproduced on a GPU) occasionally flips one int8 and moves later logits by ~1e-2.  The checks are
therefore: (1) before the first flip -- the first positions -- logits agree to 1e-5 relative
(far inside the 1e-3 bar); (2) teacher-forced over the reference's own greedy continuation, the GPU
picks the reference's token at every position whose top-2 margin exceeds the envelope that the
oracle restatement itself shows against the reference; (3) free-running greedy tokens are compared
with the oracle run in the same process."""
import os

import numpy as np
import pytest

from diolkos_b200 import synth
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


def test_tiny_logits_match_reference_golden(tiny_weights):
    w, by_name = tiny_weights
    tg = np.load(os.path.join(GOLD, "tiny.npz"))
    ps = G.TINY_PROMPTS[0]
    prompt = synth.seeded_prompt(ps, 8)
    seq = list(prompt) + list(tg[f"tokens_{ps}"])
    m = _gpu_model(synth.TINY, by_name)
    arg, top2 = tg[f"tf_argmax_{ps}"], tg[f"tf_top2_{ps}"]
    agree = 0
    for pos in range(G.TINY_TF_POSITIONS):
        lg = m.forward(int(seq[pos]), pos)
        if pos < 3:
            gl = tg[f"logits_{ps}_{pos}"]
            assert np.max(np.abs(lg - gl)) / np.max(np.abs(gl)) < 1e-5, pos
        gap = (top2[pos, 0] - top2[pos, 1]) / abs(top2[pos, 0])
        if gap > 0.03:
            assert int(np.argmax(lg)) == int(arg[pos]), pos
        agree += int(np.argmax(lg)) == int(arg[pos])
    assert agree >= G.TINY_TF_POSITIONS - 3


def test_tiny_logits_match_oracle_teacher_forced(port, tiny_weights):
    from oracle import PortModel

    w, by_name = tiny_weights
    cfg = synth.TINY
    m = _gpu_model(cfg, by_name)
    pm = PortModel(port, cfg, w)
    prompt = synth.seeded_prompt(11, 8)
    rng = np.random.default_rng(0)
    seq = list(prompt) + list(rng.integers(3, cfg.vocab_size, 40))
    errs = []
    for pos, tok in enumerate(seq):
        a = m.forward(int(tok), pos)
        b = pm.forward(int(tok), pos)
        errs.append(np.max(np.abs(a - b)) / np.max(np.abs(b)))
    assert max(errs[:3]) < 1e-5
    assert max(errs) < 5e-2, errs


def _first_near_tie(tg, ps, eps=5e-3):
    """Index of the first generated token whose position has a reference top-2 gap below eps
    (relative to the top logit): from there on any implementation may legitimately diverge."""
    top2 = tg[f"tf_top2_{ps}"]
    for pos in range(7, G.TINY_TF_POSITIONS):
        if (top2[pos, 0] - top2[pos, 1]) / abs(top2[pos, 0]) < eps:
            return pos - 7
    return G.TINY_TF_POSITIONS - 7


def test_tiny_generate_vs_reference(tiny_weights):
    """Greedy generation with the whole loop on the GPU follows the reference's own greedy tokens
    (golden) at least up to the first position where the reference's two best logits are within
    0.5% of each other."""
    w, by_name = tiny_weights
    tg = np.load(os.path.join(GOLD, "tiny.npz"))
    cfg = synth.TINY
    m = _gpu_model(cfg, by_name)
    for ps in G.TINY_PROMPTS:
        prompt = synth.seeded_prompt(ps, 8)
        gpu = m.generate(prompt, G.TINY_STEPS)
        ref = tg[f"tokens_{ps}"]
        assert len(gpu) > 0 and (gpu >= 0).all() and (gpu < cfg.vocab_size).all()
        bound = _first_near_tie(tg, ps)
        assert _first_div(gpu, ref) >= bound, (ps, bound, gpu[:20], ref[:20])


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


def test_kv_f32_and_gqa_vs_oracle(port):
    """fp32 KV cache and grouped-query attention (8 query heads per KV head, as in 70B), against
    the oracle with the same cache type; long enough to use several attention splits."""
    from oracle import PortModel, load_port_weights

    cfg = synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=1, vocab_size=2048, seq_len=512)
    w, by_name = load_port_weights(port, cfg, 77)
    for kv_f32 in (True, False):
        m = _gpu_model(cfg, by_name, kv_f32=kv_f32)
        pm = PortModel(port, cfg, w, kv_f32=kv_f32)
        rng = np.random.default_rng(1)
        seq = rng.integers(3, cfg.vocab_size, 300)
        worst = 0.0
        for pos, tok in enumerate(seq):
            a = m.forward(int(tok), pos)
            b = pm.forward(int(tok), pos)
            e = np.max(np.abs(a - b)) / np.max(np.abs(b))
            # Position 0 has no re-quantisation flip upstream yet; later positions can flip one
            # activation group (bf16 KV in particular), which moves logits by ~1e-2 relative.
            if pos == 0:
                assert e < 1e-5, (kv_f32, pos, e)
            worst = max(worst, e)
        assert worst < 5e-2, (kv_f32, worst)


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
    """dim 4096 on 256 threads takes the GEMVs' one-round-trip rmsnorm prologue (16 values per
    thread, its own sum order): logits against the oracle within the requantisation envelope, and the
    same argmax wherever the oracle's top-2 margin exceeds 3%."""
    from oracle import PortModel, load_port_weights

    cfg = synth.Config(dim=4096, hidden_dim=1024, n_layers=1, n_heads=32, n_kv_heads=8, vocab_size=1000, seq_len=64)
    w, by_name = load_port_weights(port, cfg, 91)
    m = _gpu_model(cfg, by_name, kv_f32=True)
    pm = PortModel(port, cfg, w, kv_f32=True)
    seq = np.random.default_rng(2).integers(3, cfg.vocab_size, 6)
    for pos, tok in enumerate(seq):
        a = m.forward(int(tok), pos)
        b = pm.forward(int(tok), pos)
        assert np.max(np.abs(a - b)) / np.max(np.abs(b)) < 5e-2, pos
        top = np.sort(b)[-2:]
        if top[1] - top[0] > 0.03 * abs(top[1]):
            assert int(np.argmax(a)) == int(np.argmax(b)), pos


# 32 KV heads of 32 dims: the decode attention's split count reaches its cap (ceil(5 * SMs / 32): 24 on
# 148 SMs) at position 384, where a chunk rounded up can leave the last split without positions.
CAPPED = synth.Config(dim=1024, hidden_dim=256, n_layers=2, n_heads=32, n_kv_heads=32, vocab_size=256, seq_len=600)


def test_capped_split_plan_vs_oracle(port):
    """Decode through the positions where the split count is capped (385 .. 529 had an empty last split
    under a plan that fixed the count before the chunk): finite logits within the requantisation envelope
    of the oracle at every position."""
    from oracle import PortModel, load_port_weights

    w, by_name = load_port_weights(port, CAPPED, 93)
    m = _gpu_model(CAPPED, by_name, kv_f32=True)
    pm = PortModel(port, CAPPED, w, kv_f32=True)
    seq = np.random.default_rng(3).integers(3, CAPPED.vocab_size, 560)
    worst = 0.0
    for pos, tok in enumerate(seq):
        a = m.forward(int(tok), pos)
        b = pm.forward(int(tok), pos)
        if pos >= 370:
            assert np.isfinite(a).all(), pos
            worst = max(worst, float(np.max(np.abs(a - b)) / np.max(np.abs(b))))
    assert worst < 5e-2, worst


def _logits_bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize(
    "shape,kv_f32,P",
    [
        ("tiny", False, 8),
        ("tiny", False, 200),
        ("gqa", True, 300),   # two prefill chunks (256 + 43 positions), many attention splits
        ("gqa", False, 300),
        ("wide", True, 40),   # dim 4096: the one-round-trip rmsnorm prologue
        ("capped", False, 540),  # 32 KV heads: the split count is capped (24 on 148 SMs) from position 384
        ("swiglu", True, 100),   # hidden 4096: w1|w3 (8192 rows) on the pipelined tensor-core matmul
    ],
)
def test_prefill_equals_decode_steps(port, tiny_weights, shape, kv_f32, P):
    """The batched prefill (tensor-core matmuls over the prompt positions) leaves the KV cache exactly
    as decode steps at those positions do (every model here has 2 layers or more: the prefill stops
    after the last layer's K/V rows, so only earlier layers run attention and the MLP): the logits of the last prompt position, decoded after the
    prefill, equal bit for bit those decoded after stepping every prompt position."""
    from oracle import load_port_weights

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
