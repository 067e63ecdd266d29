"""Split-KV decode across ranks (one process per GPU, long-context decode).

Each rank keeps a contiguous slice of every full-attention layer's keys in its own
KvCache, computes normalised partial attention (O_p, LSE_p) over that slice with
flash_attn_ext (RoPE positions offset by the slice start), and the partials of all
ranks are gathered and merged with attn_merge_lse:
    out = sum_p O_p exp(LSE_p - L) * sigmoid(gate),   L = log sum_p exp(LSE_p).
This is exact: softmax over the union of disjoint key sets.  The step's new row is
appended by the rank whose slice holds its position.  The gather is the only
collective; with NCCL it runs over NVLink, with gloo on the host (tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .ops import KV_PAD

GROUP = 16  # slices start on 16-token groups of the tiled cache


@dataclass(frozen=True)
class KvShard:
    """Keys [start, start + length) of the sequence live on `rank`."""

    rank: int
    world: int
    start: int
    length: int

    @property
    def capacity(self) -> int:
        """Rows of this rank's cache (padded like KvCache)."""
        return max(KV_PAD, (self.length + KV_PAD - 1) // KV_PAD * KV_PAD)

    @property
    def rope_pos_offset(self) -> int:
        return self.start

    def owns(self, pos: int) -> bool:
        return self.start <= pos < self.start + self.length

    def local_step(self, n_kv: int, q_pos0: int) -> tuple[int, int]:
        """(n_kv, q_pos0) in this slice's row numbering for a step whose sequence holds
        n_kv keys and whose first query sits at q_pos0.  Query t then sees local keys
        j <= q_pos0_local + t, i.e. global keys start + j <= q_pos0 + t; a negative
        q_pos0_local means none of this slice is visible yet (LSE -inf, weight 0)."""
        n_local = min(max(n_kv - self.start, 0), self.length)
        return n_local, q_pos0 - self.start


def plan(n_keys: int, world: int, rank: int) -> KvShard:
    """Contiguous slices of `n_keys` positions, group-aligned, as equal as possible; the
    last rank takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_keys < 1:
        raise ValueError("n_keys must be positive")
    per = (n_keys + world - 1) // world
    per = (per + GROUP - 1) // GROUP * GROUP
    start = min(rank * per, n_keys)
    length = min(per, n_keys - start)
    return KvShard(rank=rank, world=world, start=start, length=length)


def owner(n_keys: int, world: int, pos: int) -> int:
    """Rank whose slice holds position pos."""
    for r in range(world):
        if plan(n_keys, world, r).owns(pos):
            return r
    raise ValueError(f"position {pos} is outside [0, {n_keys})")


def gather(o_local: torch.Tensor, lse_local: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather the partials of every rank: o [rows][256] and lse [rows] ->
    ([world][rows][256], [world][rows]), in rank order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    o_all = torch.empty((world,) + tuple(o_local.shape), dtype=o_local.dtype, device=o_local.device)
    l_all = torch.empty((world,) + tuple(lse_local.shape), dtype=lse_local.dtype, device=lse_local.device)
    dist.all_gather(list(o_all.unbind(0)), o_local.contiguous(), group=group)
    dist.all_gather(list(l_all.unbind(0)), lse_local.contiguous(), group=group)
    return o_all, l_all
