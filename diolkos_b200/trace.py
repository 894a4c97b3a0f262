"""Per-op timeline of the persistent decode step, from its device-side stamps (dk_model_trace).

    python -m diolkos_b200.trace [--pos 200] [--layers 32] [--kv f32|bf16]

Builds the LLaMA-2-7B-shape model from seeded N(0, 0.02) weights on cuda:0 with DIOLKOS_STEP_TRACE=1,
prefills a seeded 32-token prompt, steps to position --pos and prints, for each op kind (q|k|v,
attention, wo, w1|w3, w2, and the classifier once):
  * seen:  the first CTA's sight of the op's input counter after the producing op's last CTA finished;
  * act:   the median over CTAs of input ready -> activation built;
  * cons:  the median over CTAs of activation built -> op finished (consuming the weight stages);
  * span:  from the producing op's end to this op's end (the op's share of the step).
Means over the layers, in microseconds.  The timer is the GPU's global timer (ns).
"""
from __future__ import annotations

import argparse
import ctypes as C
import os

import numpy as np

KINDS = ["qkv", "attn", "wo", "w13", "w2"]
SLOTS = 8          # stamps per (CTA, op)
READY, ACT, FIN, SEEN = 0, 1, 2, 4


def build(cfg, kv_f32: bool, seed: int):
    """The synthetic model: the same seeded weights bench.py generates, quantised on the GPU."""
    import torch

    from . import ops, synth
    from .model import Model, weight_id

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
        del w
        m.set_weight_device(which, layer, q, s)
        del q, s
    m.finalize()
    return m


def read_trace(m, n_ops_max: int, grid_max: int = 1024) -> np.ndarray:
    """[cta][op][slot] stamps of the last decode step (int64 ns, 0 = not recorded)."""
    from . import _native as N

    n = grid_max * n_ops_max * SLOTS
    buf = np.zeros(n, np.uint64)
    grid, nops = C.c_int(), C.c_int()
    N.check(N.lib().dk_model_trace(m.h, buf.ctypes.data, n, C.byref(grid), C.byref(nops)))
    G, O = grid.value, nops.value
    return buf[: G * O * SLOTS].reshape(G, O, SLOTS).astype(np.int64)


def summarise(tr: np.ndarray) -> dict:
    """Per op kind: lists of seen / act / cons / span (us) over the layers."""
    G, O, _ = tr.shape
    res = {k: {"seen": [], "act": [], "cons": [], "span": []} for k in KINDS + ["cls"]}
    prev_end = None
    for i in range(O):
        kind = "cls" if i == O - 1 else KINDS[i % 5]
        rdy, act, fin, seen = tr[:, i, READY], tr[:, i, ACT], tr[:, i, FIN], tr[:, i, SEEN]
        ran = fin > 0
        if not ran.any():
            continue
        sm = ran & (seen > 0)
        first_seen = seen[sm].min() if sm.any() else rdy[ran].min()
        am = ran & (act > 0)
        act_us = np.median((act - rdy)[am]) / 1e3 if am.any() else 0.0
        cons_us = np.median((fin - act)[am]) / 1e3 if am.any() else np.median((fin - rdy)[ran]) / 1e3
        end = fin[ran].max()
        start = prev_end if prev_end is not None else rdy[ran].min()
        res[kind]["seen"].append((first_seen - prev_end) / 1e3 if prev_end is not None else 0.0)
        res[kind]["act"].append(act_us)
        res[kind]["cons"].append(cons_us)
        res[kind]["span"].append((end - start) / 1e3)
        prev_end = end
    return res


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--pos", type=int, default=200, help="position of the traced decode step")
    ap.add_argument("--layers", type=int, default=0, help="truncate the 7B shape to this many layers")
    ap.add_argument("--kv", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--seed", type=int, default=20260, help="weights and prompt seed (bench.py's by default)")
    args = ap.parse_args()
    os.environ["DIOLKOS_STEP_TRACE"] = "1"  # read when the model is created

    import torch

    from . import synth

    torch.cuda.set_device(0)
    cfg = synth.LLAMA7B if not args.layers else synth.LLAMA7B.replace(n_layers=args.layers)
    P = 32
    if not P <= args.pos < cfg.seq_len:
        raise SystemExit(f"--pos must lie in [{P}, {cfg.seq_len})")
    m = build(cfg, args.kv == "f32", args.seed)
    prompt = synth.seeded_prompt(args.seed, P, cfg.vocab_size)
    m.set_tokens(prompt, n_forced=P)
    m.prefill(0, P - 1)
    m.enqueue_steps(P - 1, args.pos - (P - 1))  # positions 31 .. pos-1: the last step attends over pos positions
    m.sync()
    if m.device_error():
        raise SystemExit(f"device error word 0x{m.device_error():x}")
    tr = read_trace(m, cfg.n_layers * 5 + 1)
    res = summarise(tr)
    t0 = tr[:, 0, READY][tr[:, 0, READY] > 0].min()
    t1 = tr[:, :, FIN].max()
    print(f"grid {tr.shape[0]}  ops {tr.shape[1]}  step over {args.pos} positions: {(t1 - t0) / 1e3:.1f} us")
    print("op     layers   seen_us   act_us   cons_us   span_us (means per layer)")
    for k, v in res.items():
        if v["span"]:
            print(f"{k:5s} {len(v['span']):7d} {np.mean(v['seen']):9.2f} {np.mean(v['act']):8.2f} "
                  f"{np.mean(v['cons']):9.2f} {np.mean(v['span']):9.2f}")
    m.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
