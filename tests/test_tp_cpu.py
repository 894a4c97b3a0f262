"""Tensor-parallel host logic on CPU: 2, 4 and 8 gloo ranks (no GPU).

* The shard plan (diolkos_b200.tp) covers every row / column exactly once.
* Column-split partial GEMVs (wo, w2) summed over the ranks equal the full GEMV: each rank runs the
  oracle's matmul_Q8_0 on its column slice -- the slices start at multiples of 32, so the activation's
  Q8_0 groups are the reference's -- and the gloo all-reduce adds them.
* The exchange-area handshake returns every rank's handle in rank order, and a rank that never
  reaches it makes the others' handshake end with an error within the process group's timeout.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from diolkos_b200 import synth, tp

CFG = synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=1000, seq_len=64)
# divisible 8 ways: 8 heads and 8 KV heads, hidden 1024 = 8 * 128, 64 q / kv columns per rank
CFG8 = synth.Config(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=8, vocab_size=1000, seq_len=64)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_q, cfg=None):
    CFG_ = cfg or CFG
    import torch
    import torch.distributed as dist

    from oracle import Port

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        port_ = Port()
        sh = tp.shard(CFG_, rank, world)
        rng = np.random.default_rng(5)
        res = {}
        for name, n, cols in (("wo", CFG_.dim, sh.q_rows), ("w2", CFG_.hidden_dim, sh.hidden_rows)):
            d = CFG_.dim
            wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
            ws = (rng.random((d, n // 32), dtype=np.float32) * 0.01).astype(np.float32)
            x = rng.standard_normal(n).astype(np.float32)
            c0, c1 = cols
            part = port_.matmul(np.ascontiguousarray(x[c0:c1]), np.ascontiguousarray(wq[:, c0:c1]).ravel(),
                                np.ascontiguousarray(ws[:, c0 // 32:c1 // 32]).ravel(), c1 - c0, d)
            t = torch.from_numpy(part.copy())
            dist.all_reduce(t)
            full = port_.matmul(x, wq.ravel(), ws.ravel(), n, d)
            res[name] = float(np.max(np.abs(t.numpy() - full)) / np.max(np.abs(full)))
        res["handles"] = tp.exchange_handles(bytes([rank]) * 64)
        out_q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_shard_plan_covers_everything():
    for world in (1, 2):
        _covers(CFG, world)
    for world in (4, 8):
        _covers(CFG8, world)
    # the 7B and 70B shapes split 1, 2, 4 and 8 ways (heads, KV heads, hidden and vocabulary rows)
    for cfg in (synth.LLAMA7B, synth.LLAMA70B):
        for world in (1, 2, 4, 8):
            _covers(cfg, world)
    for world in (8, 16):
        with pytest.raises(ValueError):
            tp.shard(CFG, 0, world)  # 2 kv heads cannot be split 8 or 16 ways


def _covers(cfg, world):
    sh = [tp.shard(cfg, r, world) for r in range(world)]
    for field, total in (("q_rows", cfg.dim), ("kv_rows", cfg.dim * cfg.n_kv_heads // cfg.n_heads),
                         ("hidden_rows", cfg.hidden_dim), ("vocab_rows", cfg.vocab_size)):
        ranges = [getattr(s, field) for s in sh]
        assert ranges[0][0] == 0 and ranges[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        # column slices start on Q8_0 group boundaries (the activation's groups stay the reference's)
        if field in ("q_rows", "hidden_rows"):
            assert all(a % 32 == 0 for a, _ in ranges)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_split_partials_sum_to_full_gemv(world):
    cfg = CFG if world == 2 else CFG8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cfg)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in results.items():
        assert res["wo"] < 1e-5 and res["w2"] < 1e-5, (rank, res)
        assert res["handles"] == [bytes([r]) * 64 for r in range(world)]


def _handshake_worker(rank, world, port, out_q, absent):
    """Rank `absent` leaves before the exchange-area handshake; the others must get an error from it
    within the process group's timeout, not wait for good."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == absent:
        out_q.put((rank, "left"))
        time.sleep(15)  # alive but never joins: the others' collective runs out of time
        return
    t0 = time.monotonic()
    try:
        tp.exchange_handles(bytes([rank]) * 64)
        out_q.put((rank, ("completed", time.monotonic() - t0, "")))
    except Exception as e:  # the backend's timeout or connection error
        out_q.put((rank, ("error", time.monotonic() - t0, type(e).__name__)))


def test_handshake_fails_when_a_rank_never_arrives():
    world, absent = 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_handshake_worker, args=(r, world, port, q, absent)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results[absent] == "left"
    for r in range(world):
        if r != absent:
            what, seconds, _ = results[r]
            assert what == "error" and seconds < 60, results
