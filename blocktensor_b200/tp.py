"""Tensor parallelism over the GPUs of one node, one process per GPU.

The decode step's collectives run inside the persistent kernel over NVLink
(CUDA IPC mappings of every rank's exchange buffer); torch.distributed is only
the plumbing that gathers the ranks' exchange handles once, before the first
step.  Sharding (the same rule as bt_engine_create with tp_world > 1):

- q, k, v, gate and up are split by output rows: whole heads, whole KV heads,
  F / W FFN rows per rank;
- o and down are split by input columns (the rank's heads, its FFN rows),
  giving partial sums of x that the ranks add after each of them;
- the head matrix is split by vocab rows, ceil(V / W) per rank; the ranks
  agree on the greedy token;
- embeddings and norms are whole on every rank.
"""
from __future__ import annotations

from dataclasses import dataclass

MAX_WORLD = 8


@dataclass(frozen=True)
class Shard:
    heads: int
    kv_heads: int
    hidden: int          # FFN rows of this rank
    vocab: int           # head-matrix rows of this rank
    vocab0: int          # its first vocab row
    q_rows: int          # heads * head_dim
    o_cols0: int         # first input column of o-proj
    down_cols0: int      # first input column of down


def shard(vocab: int, dim: int, hidden: int, heads: int, kv_heads: int, head_dim: int,
          rank: int, world: int) -> Shard:
    """This rank's share of a model; ValueError where bt_engine_create refuses."""
    if not (1 <= world <= MAX_WORLD) or not (0 <= rank < world):
        raise ValueError("tp: rank must be < world <= 8")
    if world == 1:
        return Shard(heads, kv_heads, hidden, vocab, 0, heads * head_dim, 0, 0)
    if kv_heads % world or heads % world or (heads // world * head_dim) % 32 or hidden % (32 * world):
        raise ValueError("tp: world must divide the KV heads, and each rank's query rows and FFN rows "
                         "must be whole 32-blocks")
    vl = -(-vocab // world)
    v0 = rank * vl
    nv = min(vl, vocab - v0) if v0 < vocab else 0
    if nv == 0:
        raise ValueError("tp: world above the vocab")
    h = heads // world
    f = hidden // world
    return Shard(h, kv_heads // world, f, nv, v0, h * head_dim, rank * h * head_dim, rank * f)


def connect(engine, group=None):
    """Gathers every rank's exchange handle (torch.distributed, any backend)
    and maps them into `engine`.  Collective: every rank of `group` calls it."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if world != engine.tp_world:
        raise ValueError(f"tp.connect: process group of {world} ranks, engine built for {engine.tp_world}")
    handles = [None] * world
    dist.all_gather_object(handles, engine.tp_handle(), group=group)
    engine.tp_connect(handles)
