"""Tensor-parallel decode on 2 GPUs (one process per GPU) against the oracle.

The ranks exchange the wo / w2 partial rows inside the GEMVs over NVLink peer memory and take the
greedy token across ranks in the classifier.  Each rank runs the state-synchronised parity harness
(tests/parity.py: synced_run_tp) against the restatement (oracle/port.c, fp32 KV cache) in lockstep:
its residual stream, its slices of the attention / SwiGLU outputs and its classifier rows agree with
the oracle within 1e-3 before each step's first int8 difference, and that difference is a flip at a
rounding boundary.  Free-running greedy tokens are compared with the oracle's: both ranks agree on every
token, and a divergence from the oracle must sit at a near-tie.  Skipped with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from diolkos_b200 import synth

pytestmark = pytest.mark.gpu

CFGS = {
    "small": synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=2048, seq_len=256),
    # dim 4096 takes the GEMVs' one-round-trip reduce prologue (16 values per thread)
    "dim4096": synth.Config(dim=4096, hidden_dim=1024, n_layers=2, n_heads=32, n_kv_heads=8, vocab_size=2048,
                            seq_len=256),
}
SEED, STEPS = 77, 48


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out_q, cfg_name, kv_f32=True):
    CFG = CFGS[cfg_name]
    import torch.distributed as dist

    from diolkos_b200 import tp
    from diolkos_b200.model import Model
    from oracle import PW_RMS_ATT, PW_RMS_FFN, PW_RMS_FINAL, Port, PortModel, load_port_weights
    from tests import parity

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        port_ = Port()
        w, by_name = load_port_weights(port_, CFG, SEED)
        m = Model(CFG, kv_f32=kv_f32, device=rank, tp_rank=rank, tp_world=world)
        m.load_named(by_name)
        tp.connect(m)
        m.finalize()
        prompt = synth.seeded_prompt(3, 8, CFG.vocab_size)
        toks = m.generate(prompt, STEPS)
        m.dump_enable()
        norms = []
        for l in range(CFG.n_layers):
            norms += [np.asarray(w[(PW_RMS_ATT, l)], np.float32), None, np.asarray(w[(PW_RMS_FFN, l)], np.float32), None]
        norms.append(np.asarray(w[(PW_RMS_FINAL, -1)], np.float32))
        seq = list(prompt) + list(np.random.default_rng(4).integers(3, CFG.vocab_size, 32))
        recs = parity.synced_run_tp(m, PortModel(port_, CFG, w, kv_f32=kv_f32), seq, len(seq), port_, norms, CFG,
                                    rank, world)
        # teacher-forced (not synchronised) along the oracle's greedy stream: this rank's logit rows
        ref_toks = PortModel(port_, CFG, w, kv_f32=kv_f32).generate(prompt, STEPS)
        tf_seq = list(prompt) + list(ref_toks)
        m.dump_enable(False)
        tf = np.stack([m.forward(int(tf_seq[p]), p) for p in range(min(len(tf_seq), STEPS))])
        err = m.device_error()
        m.close()
        try:
            summ = parity.check_tp(recs, f"tp{world} {cfg_name} {'fp32' if kv_f32 else 'bf16'} KV rank {rank}")
        except AssertionError as e:
            summ = f"FAILED: {e}"
        out_q.put((rank, toks, summ, err, tf))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kv_f32", [True, False])
@pytest.mark.parametrize("cfg_name", sorted(CFGS))
def test_tp2_vs_oracle(cfg_name, kv_f32):
    CFG = CFGS[cfg_name]
    from oracle import Port, PortModel, load_port_weights

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, cfg_name, kv_f32)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, toks, summ, err, tf = q.get(timeout=600)
        res[r] = (toks, summ, err, tf)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(res[r][2] == 0 for r in res), {r: res[r][2] for r in res}
    for r in res:
        assert not res[r][1].startswith("FAILED"), res[r][1]
        print(res[r][1])
    np.testing.assert_array_equal(res[0][0], res[1][0])  # the ranks agree on every token
    # free-running greedy tokens against the oracle's; a divergence must be a near-tie
    port_ = Port()
    w, _ = load_port_weights(port_, CFG, SEED)
    prompt = synth.seeded_prompt(3, 8, CFG.vocab_size)
    ref_toks = PortModel(port_, CFG, w, kv_f32=kv_f32).generate(prompt, STEPS)
    gpu = res[0][0]
    n = min(len(ref_toks), len(gpu))
    first_div = next((i for i in range(n) if ref_toks[i] != gpu[i]), n)
    print(f"tp{world} {cfg_name}: {first_div} identical greedy tokens of {n}")
    if first_div < n:
        # the histories agree up to the divergence: the oracle's margin between its token and the GPU's must
        # lie within the measured GPU-vs-oracle logit difference there (a near-tie)
        pm = PortModel(port_, CFG, w, kv_f32=kv_f32)
        seq = list(prompt) + list(ref_toks)
        p_div = len(prompt) - 1 + first_div
        for pos in range(p_div + 1):
            lo = pm.forward(int(seq[pos]), pos)
        lg = np.where(np.isnan(res[0][3][p_div]), res[1][3][p_div], res[0][3][p_div])  # both ranks' rows
        a_ref, a_gpu = int(ref_toks[first_div]), int(gpu[first_div])
        margin, diff = float(lo[a_ref] - lo[a_gpu]), float(np.max(np.abs(lg - lo)))
        assert margin <= 2.0 * diff, (first_div, margin, diff)


def _rank_prefill(rank, world, port, out_q, cfg_name, kv_f32=True):
    CFG = CFGS[cfg_name]
    import torch.distributed as dist

    from diolkos_b200 import tp
    from diolkos_b200.model import Model
    from oracle import Port, load_port_weights

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _, by_name = load_port_weights(Port(), CFG, SEED)
        m = Model(CFG, kv_f32=kv_f32, device=rank, tp_rank=rank, tp_world=world)
        m.load_named(by_name)
        tp.connect(m)
        m.finalize()
        P = 40
        prompt = synth.seeded_prompt(5, P, CFG.vocab_size)
        m.set_tokens(prompt, n_forced=P)
        m.prefill(0, P - 1)
        after = m.forward(int(prompt[P - 1]), P - 1)
        for pos in range(P):
            stepped = m.forward(int(prompt[pos]), pos)
        gen = m.generate(prompt[:12], STEPS)
        os.environ["DIOLKOS_PREFILL"] = "0"
        gen_stepped = m.generate(prompt[:12], STEPS)
        del os.environ["DIOLKOS_PREFILL"]
        err = m.device_error()
        m.close()
        out_q.put((rank, after, stepped, gen, gen_stepped, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kv_f32", [True, False])
@pytest.mark.parametrize("cfg_name", sorted(CFGS))
def test_tp2_prefill_equals_stepped_decode(cfg_name, kv_f32):
    """Tensor-parallel prefill: the wo / w2 partial rows of a chunk cross NVLink and are summed in rank
    order, as the decode step sums them; so the KV cache after a prefill is the one stepped decode leaves
    on every rank (bit-exact logits of this rank's classifier rows after it), and generate gives the same
    tokens with and without the prefill."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_prefill, args=(r, world, port, q, cfg_name, kv_f32)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, after, stepped, gen, gen_stepped, err = q.get(timeout=300)
        res[r] = (after, stepped, gen, gen_stepped, err)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, (after, stepped, gen, gen_stepped, err) in res.items():
        assert err == 0, (r, err)
        rows = ~np.isnan(stepped)  # this rank's classifier rows
        assert rows.any()
        np.testing.assert_array_equal(after[rows].view(np.uint32), stepped[rows].view(np.uint32))
        assert len(gen) > 0
        np.testing.assert_array_equal(gen, gen_stepped)
