"""Tensor-parallel sharding of the decode path by KV head (one process per GPU).

The task table is head-independent (records are (request, split)), so N GPUs split the
work with no exchange step: rank i owns KV heads [i*Hkv/N, (i+1)*Hkv/N), the matching
query heads (each KV head serves ``group`` consecutive query heads) and its slice of
every layer's KV pool, and builds its own plan with ``kv_heads = Hkv/N`` tasks per
record.  Gathering the per-rank outputs along the head dimension gives the unsharded
output; that reassembly belongs to the model (its o_proj all-reduce), not to this path.
"""
from __future__ import annotations

import dataclasses

from .config import DecodeConfig


@dataclasses.dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_offset: int          # first KV head owned by this rank
    kv_heads: int           # KV heads owned by this rank
    q_offset: int           # first query head owned by this rank
    query_heads: int        # query heads owned by this rank


def head_shard(config: DecodeConfig, rank: int, world: int) -> HeadShard:
    """The KV / query head range of ``rank`` out of ``world`` (KV heads must divide evenly)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if config.kv_heads % world:
        raise ValueError(f"{config.kv_heads} KV heads do not shard evenly over {world} GPUs")
    hkv = config.kv_heads // world
    g = config.group_size
    return HeadShard(rank, world, rank * hkv, hkv, rank * hkv * g, hkv * g)


def shard_config(config: DecodeConfig, shard: HeadShard) -> DecodeConfig:
    """The per-GPU capture configuration: same capacities, the shard's head counts."""
    return dataclasses.replace(config, query_heads=shard.query_heads, kv_heads=shard.kv_heads)


def shard_q(q, shard: HeadShard):
    """Query rows of the shard: q[:, q_offset : q_offset + query_heads]."""
    return q[:, shard.q_offset:shard.q_offset + shard.query_heads]


def shard_kv(kv, shard: HeadShard):
    """KV pool slice of the shard along the head axis ([..., Hkv, D] -> [..., Hkv/N, D])."""
    return kv[..., shard.kv_offset:shard.kv_offset + shard.kv_heads, :]


def assemble(outputs):
    """Concatenate per-rank outputs [B, Hq/N, D] (rank order) into [B, Hq, D]."""
    import torch
    return torch.cat(list(outputs), dim=1)
