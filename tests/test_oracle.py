"""The oracle (oracle/port.c) pinned against the reference: the committed golden fixtures (outputs
of the compiled reference, tests/golden/make_golden.py) and, where oracle/_ref is built, the
compiled reference itself on fresh inputs.  CPU only."""
import hashlib
import os
import tempfile

import numpy as np
import pytest

from diolkos_b200 import synth
from tests.golden import make_golden as G

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def kgold():
    return np.load(os.path.join(GOLD, "kernels.npz"))


@pytest.fixture(scope="module")
def tgold():
    return np.load(os.path.join(GOLD, "tiny.npz"))


@pytest.mark.parametrize("case", G.QUANT_F32_CASES)
def test_port_quant_f32_matches_golden(port, kgold, case):
    seed, n, sc = case
    q, s = port.quant_f32(G.quant_f32_input(seed, n, sc))
    assert sha(q) == str(kgold[f"qf32_{seed}_q"])
    assert sha(s) == str(kgold[f"qf32_{seed}_s"])


@pytest.mark.parametrize("case", G.QUANT_BF16_CASES)
def test_port_quant_bf16_matches_golden(port, kgold, case):
    seed, n, sc = case
    q, s = port.quant_bf16(G.quant_bf16_input(seed, n, sc))
    assert sha(q) == str(kgold[f"qbf16_{seed}_q"])
    assert sha(s) == str(kgold[f"qbf16_{seed}_s"])


@pytest.mark.parametrize("case", G.GEMV_CASES)
def test_port_gemv_bit_exact_with_golden(port, kgold, case):
    n, d, seed = case
    wb, x = G.gemv_inputs(n, d, seed)
    wq, ws = port.quant_bf16(wb)
    out = port.matmul(x, wq, ws, n, d)
    np.testing.assert_array_equal(out.view(np.uint32), kgold[f"gemv_{n}x{d}"].view(np.uint32))


def test_port_quant_round_half_even_and_edges(port):
    # exact .5 products: amax 127 -> scale 127*(1/127f), values chosen on half steps
    x = np.zeros(64, np.float32)
    x[:32] = np.linspace(-127, 127, 32, dtype=np.float32)
    x[32] = 2.5; x[33] = 3.5; x[34] = -2.5; x[63] = 127.0
    q, s = port.quant_f32(x)
    inv = np.float32(1.0) / s
    expect = np.rint(x * np.repeat(inv, 32)).astype(np.int8)  # numpy rint rounds half to even
    np.testing.assert_array_equal(q, expect)
    # an all-zero group has scale 0 and quantises to 0 (the reference's cast of NaN is undefined)
    qz, sz = port.quant_f32(np.zeros(32, np.float32))
    assert sz[0] == 0.0 and not qz.any()


def test_port_vs_reference_live_quant_and_gemv(port, ref):
    rng = np.random.default_rng(99)
    x = rng.standard_normal(32 * 5000, dtype=np.float32) * np.float32(7.0)
    for a, b in zip(port.quant_f32(x), ref.quant_f32(x)):
        np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))
    wb = synth.f32_to_bf16_bits(rng.standard_normal(32 * 6000, dtype=np.float32) * np.float32(0.02))
    for a, b in zip(port.quant_bf16(wb), ref.quant_bf16(wb)):
        np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))
    n, d = 1024, 96
    wq, ws = port.quant_bf16(synth.f32_to_bf16_bits(rng.standard_normal(n * d, dtype=np.float32) * np.float32(0.02)))
    xv = rng.standard_normal(n, dtype=np.float32)
    np.testing.assert_array_equal(port.matmul(xv, wq, ws, n, d).view(np.uint32),
                                  ref.matmul(xv, wq, ws, n, d).view(np.uint32))


@pytest.mark.parametrize("n,d", [(8192, 64), (28672, 32), (11008, 48), (32, 33)])
def test_port_vs_reference_live_gemv_widths(port, ref, n, d):
    """The restatement's GEMV against the compiled reference at the 70B shape's input widths (dim 8192,
    hidden 28672), the 7B hidden width and the narrowest input: bit for bit."""
    rng = np.random.default_rng(n + d)
    wq, ws = port.quant_bf16(synth.f32_to_bf16_bits(rng.standard_normal(n * d, dtype=np.float32) * np.float32(0.02)))
    xv = rng.standard_normal(n, dtype=np.float32)
    np.testing.assert_array_equal(port.matmul(xv, wq, ws, n, d).view(np.uint32),
                                  ref.matmul(xv, wq, ws, n, d).view(np.uint32))


def test_port_group_dots_exact(port):
    rng = np.random.default_rng(5)
    n, d = 256, 7
    xq = rng.integers(-127, 128, n, dtype=np.int8)
    wq = rng.integers(-127, 128, n * d, dtype=np.int8)
    dots = port.group_dots(xq, wq, n, d)
    ref = (wq.reshape(d, n // 32, 32).astype(np.int64) * xq.reshape(n // 32, 32).astype(np.int64)).sum(-1)
    np.testing.assert_array_equal(dots, ref)


def test_port_rmsnorm_softmax_vs_reference(port, ref):
    rng = np.random.default_rng(6)
    for n in (4096, 11008):
        x = rng.standard_normal(n, dtype=np.float32)
        w = rng.standard_normal(n, dtype=np.float32)
        # same 8-lane order as the compiled reference; the 1/sqrt may differ in its last bit
        np.testing.assert_allclose(port.rmsnorm(x, w), ref.rmsnorm(x, w), rtol=3e-7, atol=0)
    s = rng.standard_normal(300, dtype=np.float32)
    np.testing.assert_allclose(port.softmax(s), ref.softmax(s), rtol=1e-6, atol=1e-9)


def test_port_sampler_matches_reference(port, ref):
    rng = np.random.default_rng(8)
    logits = rng.standard_normal(32000, dtype=np.float32) * np.float32(3.0)
    assert port.argmax(logits) == ref.argmax(logits)
    ties = np.zeros(100, np.float32)
    ties[[17, 40]] = 5.0
    assert port.argmax(ties) == ref.argmax(ties) == 17
    for t, p in [(1.0, 0.9), (0.7, 1.0), (1.3, 0.5)]:
        st_p = st_r = 12345
        for _ in range(20):
            tp, st_p = port.sample(logits, t, p, st_p)
            tr, st_r = ref.sample(logits, t, p, st_r)
            assert tp == tr and st_p == st_r


def _first_div(a, b):
    m = min(len(a), len(b))
    for i in range(m):
        if a[i] != b[i]:
            return i
    return m


def test_port_tiny_model_vs_golden(port, tgold):
    """Teacher-forced logits of the restatement against the reference's: bit-close before the
    first activation-requantisation flip, and the same argmax wherever the reference's top-2 gap
    exceeds the measured port-vs-reference logit envelope."""
    from oracle import PortModel, load_port_weights

    cfg = synth.TINY
    w, _ = load_port_weights(port, cfg, G.TINY_SEED)
    ps = G.TINY_PROMPTS[0]
    prompt = synth.seeded_prompt(ps, 8)
    toks = tgold[f"tokens_{ps}"]
    seq = list(prompt) + list(toks)
    m = PortModel(port, cfg, w)
    arg, top2 = tgold[f"tf_argmax_{ps}"], tgold[f"tf_top2_{ps}"]
    for pos in range(G.TINY_TF_POSITIONS):
        lg = m.forward(int(seq[pos]), pos)
        if pos < 3:
            gl = tgold[f"logits_{ps}_{pos}"]
            assert np.max(np.abs(lg - gl)) / np.max(np.abs(gl)) < 1e-5
        gap = (top2[pos, 0] - top2[pos, 1]) / abs(top2[pos, 0])
        if gap > 0.03:
            assert int(np.argmax(lg)) == int(arg[pos]), pos
    # free-running greedy: the restatement follows the reference for the first tokens
    gen = PortModel(port, cfg, w).generate(prompt, G.TINY_STEPS)
    assert _first_div(gen, toks) >= 8


def test_reference_native_build(ref):
    """The reference's -march=native build follows the portable build up to the order of its fp32
    sums, which depends on the host CPU: quantised bytes are identical, logits agree within the
    activation-requantisation envelope (and are identical on hosts whose native vector shape is the
    portable one)."""
    from oracle import Ref, ref_path

    if ref_path("portable") is None or ref_path("native") is None:
        pytest.skip("both reference variants are needed")
    a, b = Ref("native"), Ref("portable")
    rng = np.random.default_rng(12)
    x = rng.standard_normal(32 * 2000, dtype=np.float32)
    for u, v in zip(a.quant_f32(x), b.quant_f32(x)):
        np.testing.assert_array_equal(u.view(np.uint8), v.view(np.uint8))
    tmp = tempfile.mkdtemp()
    md = os.path.join(tmp, "tiny")
    synth.write_model(md, synth.TINY, G.TINY_SEED)
    ma, mb = a.load(md, tmp), b.load(md, tmp)
    prompt = synth.seeded_prompt(7, 8)
    for pos in range(6):
        la, lb = ma.forward(int(prompt[pos]), pos), mb.forward(int(prompt[pos]), pos)
        assert np.max(np.abs(la - lb)) / np.max(np.abs(lb)) < 5e-2


def test_hooked_reference_checkpoints(ref):
    """The hooked reference build (oracle/ref_hooks.c: the unmodified transformer.c with its rmsnorm /
    matmul calls routed through recording hooks) computes exactly what the plain build computes --
    logits and KV rows bit-identical over several positions -- and its checkpoints are the reference's
    own values: each recorded activation is rmsnorm(recorded residual) for the norm prologues and
    the reference quantiser's output of the recorded input, bit for bit."""
    from oracle import Ref, ref_path

    if ref_path("portable", hooked=True) is None:
        pytest.skip("the hooked reference build is not present")
    hk = Ref("portable", hooked=True)
    plain = Ref("portable")
    cfg = synth.TINY
    tmp = tempfile.mkdtemp()
    md = os.path.join(tmp, "tiny")
    synth.write_model(md, cfg, G.TINY_SEED)
    mh, mp = hk.load(md, tmp), plain.load(md, tmp)
    prompt = synth.seeded_prompt(7, 8)
    w_att = np.ones(cfg.dim, np.float32)  # the synthetic models' norm weights are 1.0
    L = cfg.n_layers
    for pos in range(6):
        tok = int(prompt[pos])
        lh, xres, acts = mh.forward_dump(tok, pos)
        lp = mp.forward(tok, pos)
        np.testing.assert_array_equal(lh.view(np.uint32), lp.view(np.uint32))
        assert xres.shape == (2 * L + 1, cfg.dim) and len(acts) == 4 * L + 1
        for l in range(L):
            for k, xi in ((0, 2 * l), (2, 2 * l + 1)):
                np.testing.assert_array_equal(acts[4 * l + k][0].view(np.uint32),
                                              plain.rmsnorm(xres[xi], w_att).view(np.uint32))
        np.testing.assert_array_equal(acts[4 * L][0].view(np.uint32), plain.rmsnorm(xres[2 * L], w_att).view(np.uint32))
        for ain, aq, asc in acts:
            q, s = plain.quant_f32(ain)
            np.testing.assert_array_equal(aq, q)
            np.testing.assert_array_equal(asc.view(np.uint32), s.view(np.uint32))
    for l in (0, L - 1):
        for a, b in zip(mh.kv_rows(l, 0, 6), mp.kv_rows(l, 0, 6)):
            np.testing.assert_array_equal(a, b)
