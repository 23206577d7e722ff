"""KV-head sharding of batch decode across the GPUs of one box.

Attention for KV head h reads only that head's pages and only Q heads
[h*G, (h+1)*G) with G = q_heads / kv_heads (the GQA adjacency of the
reference: src/v2/paged_attention.cu:122, src/v2/reference_attention.cpp:58).
So rank g of N owns KV heads [g*Hkv/N, (g+1)*Hkv/N) with their own page pool,
storage and block tables, and Q heads [g*Hq/N, (g+1)*Hq/N); token counts are
the same on every rank, page ids are not. The decode itself needs no
exchange. Outputs are all-gathered (NCCL over NVLink on GPUs, gloo in the CPU
tests) only to verify, then reordered from [rank][batch][Hq/N][hd] to
[batch][Hq][hd].
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_begin: int
    kv_end: int
    q_begin: int
    q_end: int

    @property
    def kv_heads(self) -> int:
        return self.kv_end - self.kv_begin

    @property
    def q_heads(self) -> int:
        return self.q_end - self.q_begin


def shard_heads(kv_heads: int, q_heads: int, world: int, rank: int) -> HeadShard:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    if kv_heads % world != 0:
        raise ValueError(f"{kv_heads} KV heads cannot be split evenly over {world} ranks")
    if q_heads % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    per = kv_heads // world
    group = q_heads // kv_heads
    return HeadShard(rank, world, rank * per, (rank + 1) * per, rank * per * group, (rank + 1) * per * group)


def assemble(gathered, batch: int, q_heads: int, head_size: int):
    """Rank-ordered list of per-rank outputs [batch][q_heads/N][hd] -> [batch][q_heads][hd]."""
    world = len(gathered)
    per = q_heads // world
    parts = [g.reshape(batch, per, head_size) for g in gathered]
    try:
        import torch

        if isinstance(parts[0], torch.Tensor):
            return torch.cat(parts, dim=1)
    except ImportError:  # pragma: no cover
        pass
    import numpy as np

    return np.concatenate(parts, axis=1)
