"""Head-parallel sharding of a Gated DeltaNet layer across the GPUs of one box.

Key head i serves value heads i*r .. i*r+r-1 (r = Hv / Hk, repeat_interleave
in python/qwen35.py:592-594), so splitting the 16 key heads into N contiguous
groups splits the 48 value heads into N contiguous groups with no head
shared between ranks.  Everything of the layer between its projections is
per head -- the conv channels of those heads, the gates, the state, the
recurrence and the gated norm -- so a rank runs its shard with no
communication, and the only collective is one all-gather of the normed head
outputs at the layer boundary (before out_proj).

Channel layout of the conv input (cpp/src/model.cpp:592-596): contiguous
[q (Hk*Dk) | k (Hk*Dk) | v (Hv*Dv)].
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    k0: int          # first key head
    k1: int          # one past the last key head
    v0: int          # first value head
    v1: int

    @property
    def hk(self) -> int:
        return self.k1 - self.k0

    @property
    def hv(self) -> int:
        return self.v1 - self.v0


def head_shard(rank: int, world: int, Hk: int = 16, Hv: int = 48) -> HeadShard:
    """Key heads [Hk*rank/world, Hk*(rank+1)/world) and their value heads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if Hk % world or Hv % Hk:
        raise ValueError(f"Hk={Hk} must divide by world={world} and Hv={Hv} by Hk")
    r = Hv // Hk
    k0, k1 = Hk * rank // world, Hk * (rank + 1) // world
    return HeadShard(rank, world, k0, k1, k0 * r, k1 * r)


def conv_channels(sh: HeadShard, Hk: int = 16, Dk: int = 128, Dv: int = 128) -> List[range]:
    """The conv-input channel ranges of this shard, in [q | k | v] order."""
    q = range(sh.k0 * Dk, sh.k1 * Dk)
    k = range(Hk * Dk + sh.k0 * Dk, Hk * Dk + sh.k1 * Dk)
    v = range(2 * Hk * Dk + sh.v0 * Dv, 2 * Hk * Dk + sh.v1 * Dv)
    return [q, k, v]


def channel_index(sh: HeadShard, Hk: int = 16, Dk: int = 128, Dv: int = 128) -> List[int]:
    """Flat list of this shard's conv channels, in the shard's own [q|k|v] order."""
    out: List[int] = []
    for r in conv_channels(sh, Hk, Dk, Dv):
        out.extend(r)
    return out


def assemble(parts, axis_heads: int = -2):
    """Per-rank head blocks (rank order) -> the full head axis.  Works for
    numpy arrays and torch tensors whose head axis is `axis_heads`."""
    first = parts[0]
    if hasattr(first, "cpu") and hasattr(first, "dim"):        # torch
        import torch
        return torch.cat(list(parts), dim=axis_heads)
    import numpy as np
    return np.concatenate(list(parts), axis=axis_heads)
