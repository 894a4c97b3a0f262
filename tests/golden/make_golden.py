"""Generate the golden fixtures in this directory from the compiled reference (oracle/_ref).

The reference ships no known-answer tests for its Q8_0 path, so the fixtures are outputs of the
reference itself: its unmodified C sources compiled with its own -Ofast flags (oracle/Makefile,
target `ref`) and driven through oracle/ref_driver.c.  Inputs are regenerated from seeds
(numpy PCG64), so only the outputs are stored.

Run here, where the reference tree exists:
    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from diolkos_b200 import synth  # noqa: E402
from oracle import Ref  # noqa: E402

# Inputs of the quantiser cases (regenerated identically by the tests).
QUANT_F32_CASES = [(11, 32 * 4096, 1.0), (12, 32 * 1024, 1e-3), (13, 32 * 1024, 1e4)]
QUANT_BF16_CASES = [(21, 32 * 8192, 0.02), (22, 32 * 1024, 3.0)]
GEMV_CASES = [(4096, 256, 31), (11008, 128, 32), (288, 768, 33), (768, 288, 34), (4096, 32, 35)]
TINY_SEED = 1234
TINY_PROMPTS = [7, 8, 9]
TINY_STEPS = 8 + 128
TINY_TF_POSITIONS = 8 + 64


def quant_f32_input(seed, n, scale):
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal(n, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def quant_bf16_input(seed, n, scale):
    rng = np.random.Generator(np.random.PCG64(seed))
    return synth.f32_to_bf16_bits(rng.standard_normal(n, dtype=np.float32) * np.float32(scale))


def gemv_inputs(n, d, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    wb = synth.f32_to_bf16_bits(rng.standard_normal(n * d, dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(n, dtype=np.float32)
    return wb, x


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ref = Ref()
    out = {}
    for seed, n, sc in QUANT_F32_CASES:
        q, s = ref.quant_f32(quant_f32_input(seed, n, sc))
        out[f"qf32_{seed}_q"] = sha(q)
        out[f"qf32_{seed}_s"] = sha(s)
        out[f"qf32_{seed}_head"] = q[:64].copy()
    for seed, n, sc in QUANT_BF16_CASES:
        q, s = ref.quant_bf16(quant_bf16_input(seed, n, sc))
        out[f"qbf16_{seed}_q"] = sha(q)
        out[f"qbf16_{seed}_s"] = sha(s)
        out[f"qbf16_{seed}_head"] = q[:64].copy()
    for n, d, seed in GEMV_CASES:
        wb, x = gemv_inputs(n, d, seed)
        wq, ws = ref.quant_bf16(wb)
        out[f"gemv_{n}x{d}"] = ref.matmul(x, wq, ws, n, d)
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **{k: np.asarray(v) for k, v in out.items()})

    cfg = synth.TINY
    tmp = tempfile.mkdtemp()
    mdir = os.path.join(tmp, "tiny")
    synth.write_model(mdir, cfg, TINY_SEED)
    model = {}
    for ps in TINY_PROMPTS:
        prompt = synth.seeded_prompt(ps, 8)
        toks, _ = ref.load(mdir, tmp).generate(prompt, TINY_STEPS)
        model[f"tokens_{ps}"] = toks
        m = ref.load(mdir, tmp)
        seq = list(prompt) + list(toks)
        top = np.zeros((TINY_TF_POSITIONS, 2), np.float32)
        arg = np.zeros(TINY_TF_POSITIONS, np.int32)
        for pos in range(min(TINY_TF_POSITIONS, len(seq))):
            lg = m.forward(int(seq[pos]), pos)
            o = np.argsort(-lg, kind="stable")
            arg[pos] = o[0]
            top[pos] = lg[o[:2]]
            if ps == TINY_PROMPTS[0] and pos < 3:
                model[f"logits_{ps}_{pos}"] = lg
        model[f"tf_argmax_{ps}"] = arg
        model[f"tf_top2_{ps}"] = top
    np.savez_compressed(os.path.join(HERE, "tiny.npz"), **model)
    print("wrote", os.path.join(HERE, "kernels.npz"), os.path.join(HERE, "tiny.npz"))


if __name__ == "__main__":
    main()
