"""bench.py's checks on CPU (no GPU): the free-running comparison and the teacher-forced agreement with a
reference stream, on a fake model, at 1 and 2 gloo ranks (tensor parallel: each rank sees only its
classifier rows); and the byte accounting behind the roofline fractions."""
import os
import socket
import sys

import numpy as np
import torch.multiprocessing as mp

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402

V = 50


class FakeModel:
    """Logits of position pos: a seeded vector whose largest entry is `(7 * pos) % V`, except at the
    positions in `tie`, where entries `(7 * pos) % V` and `(7 * pos + 1) % V` tie and the larger index
    carries a 1e-6 relative excess.  Rank r of w holds rows [r * V / w, (r + 1) * V / w), NaN elsewhere."""

    def __init__(self, rank=0, world=1, tie=()):
        self.rank, self.world, self.tie = rank, world, set(tie)

    def forward(self, token, pos):
        lg = np.random.default_rng(pos).random(V).astype(np.float32)
        a = (7 * pos) % V
        lg[a] = 5.0
        if pos in self.tie:
            lg[(a + 1) % V] = np.float32(5.0 * (1 + 1e-6))
        per = V // self.world
        out = np.full(V, np.nan, np.float32)
        out[self.rank * per:(self.rank + 1) * per] = lg[self.rank * per:(self.rank + 1) * per]
        return out


def _ref_stream(P, G):
    """The reference's greedy tokens of positions P-1 .. P-2+G under FakeModel without ties."""
    return [(7 * pos) % V for pos in range(P - 1, P - 1 + G)]


def test_token_check_counts_to_first_divergence():
    r = bench.token_check([1, 2, 3, 9], [1, 2, 3, 4], [[1.0, 0.9]] * 4, "x")
    assert r["identical"] == 3 and r["first_divergence"] == 3 and abs(r["ref_top2_gap_at_divergence"] - 0.1) < 1e-6


def test_forced_check_single_rank():
    P, G = 5, 20
    prompt = list(range(P))
    ref = _ref_stream(P, G)
    top2 = [[5.0, 4.9]] * G
    tie_pos = P - 1 + 6  # generated index 6
    r = bench.forced_check(FakeModel(tie=[tie_pos]), prompt, ref, top2, 1, "fake")
    assert r["of"] == G and r["agree"] == G - 1
    (d,) = r["disagreements"]
    assert d["index"] == 6 and d["ref"] == ref[6] and d["gpu"] == (ref[6] + 1) % V
    assert 0 < d["gpu_gap"] < 1e-5 and abs(d["ref_top2_gap"] - 0.02) < 1e-6


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P, G = 5, 20
        ref = _ref_stream(P, G)
        # a tie across ranks (row 49 on rank 1 against row 0 on rank 0) and one inside rank 0 (rows 20, 21)
        ties = [p for p in range(P - 1, P - 1 + G) if (7 * p) % V in (49, 20)]
        r = bench.forced_check(FakeModel(rank, world, tie=ties), list(range(P)), ref, None, world, "fake")
        out_q.put((rank, r, ties))
    finally:
        dist.destroy_process_group()


def test_forced_check_two_ranks_gathers_the_global_choice():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, r0, ties), (_, r1, _) = sorted(res, key=lambda t: t[0])
    assert r0 == r1  # every rank reports the same result
    P, G = 5, 20
    ref = _ref_stream(P, G)
    assert len(ties) == 2 and r0["agree"] == G - len(ties)
    for d in r0["disagreements"]:
        assert d["gpu"] == (d["ref"] + 1) % V and 0 < d["gpu_gap"] < 1e-5
        assert "ref_top2_gap" not in d
    assert sorted(d["index"] for d in r0["disagreements"]) == [p - (P - 1) for p in ties]


def test_roofline_byte_accounting():
    """The algorithmic bytes behind the roofline fractions: the 7B-shape weights once per token at 1.125 B
    per value (6.607 G matmul values -> 7.433 GB, plus activations, norms and one embedding row), the KV
    rows 2 * L * (pos + 1) * kv_dim * element size, and the GEMV shapes' d*n*1.125 + n*1.125 + d*4."""
    from diolkos_b200 import synth

    cfg = synth.LLAMA7B
    mat_values = cfg.n_layers * (4 * cfg.dim * cfg.dim + 3 * cfg.hidden_dim * cfg.dim) + cfg.vocab_size * cfg.dim
    assert mat_values == 6_607_077_376
    wb = bench.weight_bytes_per_token(cfg)
    gemvs = [(cfg.dim, cfg.dim), (cfg.kv_dim, cfg.dim), (cfg.kv_dim, cfg.dim), (cfg.dim, cfg.dim),
             (cfg.hidden_dim, cfg.dim), (cfg.dim, cfg.hidden_dim), (cfg.hidden_dim, cfg.dim)]
    want = (cfg.n_layers * (sum(bench.gemv_alg_bytes(d, n) for d, n in gemvs) + 2 * cfg.dim * 4)
            + bench.gemv_alg_bytes(cfg.vocab_size, cfg.dim) + cfg.dim * 1.125 + cfg.dim * 4)
    assert wb == want
    assert 0 < wb - mat_values * 1.125 < 10e6, wb  # activations, outputs, norms, one embedding row
    assert bench.kv_bytes_read(cfg, 0, 1, 4) == 2 * 32 * 4096 * 4
    # the decode workload: 256 tokens at positions 31 .. 286, fp32 KV
    kv = bench.kv_bytes_read(cfg, 31, 287, 4)
    assert kv == 2.0 * 32 * 4096 * 4 * sum(p + 1 for p in range(31, 287))
    assert abs((wb + kv / 256) / 1e9 - 7.608) < 0.001  # the step roofline's bytes per token
    assert bench.gemv_alg_bytes(4096, 4096) == 4096 * 4096 * 1.125 + 4096 * 1.125 + 4096 * 4
    assert abs(bench.gemv_alg_bytes(32000, 4096) / 1e6 - 147.59) < 0.01
