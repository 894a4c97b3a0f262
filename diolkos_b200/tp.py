"""Tensor-parallel plumbing on the host: the shard plan and the exchange-area handshake.

The split follows the reference's client/worker topology (src/bin/client.c), one rank per GPU of one
node: rank r of `world` holds attention heads [r*H/world, (r+1)*H/world) (and the matching KV heads),
w1/w3 rows [r*hidden/world, ...), the same columns of w2 and the matching columns of wo, and the
classifier rows [r*ceil(V/world), ...).  The engine (dk_model_create) cuts these slices out of the full
matrices itself; this module states the plan for tests and tools, and connects the ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import synth


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    q_rows: tuple      # rows of wq (= columns of wo) held by this rank
    kv_rows: tuple     # rows of wk / wv
    hidden_rows: tuple # rows of w1 / w3 (= columns of w2)
    vocab_rows: tuple  # rows of the classifier


def shard(cfg: synth.Config, rank: int, world: int) -> Shard:
    """This rank's slices, as (start, stop) ranges of the full matrices."""
    hs = cfg.dim // cfg.n_heads
    if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.hidden_dim % (32 * world) or \
            (hs * cfg.n_heads // world) % 32:
        raise ValueError(f"{world} ranks do not divide this model evenly")
    qd = hs * cfg.n_heads // world
    kd = hs * cfg.n_kv_heads // world
    hd = cfg.hidden_dim // world
    per = -(-cfg.vocab_size // world)
    v0 = min(cfg.vocab_size, rank * per)
    return Shard(rank, world, (rank * qd, (rank + 1) * qd), (rank * kd, (rank + 1) * kd),
                 (rank * hd, (rank + 1) * hd), (v0, min(cfg.vocab_size, v0 + per)))


def exchange_handles(handle: bytes, group=None) -> list:
    """All ranks' exchange-area handles in rank order (torch.distributed all_gather_object)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def connect(model, group=None) -> None:
    """Share the ranks' exchange areas and map them into this rank's model (before finalize)."""
    model.comm_connect(exchange_handles(model.comm_handle(), group))
