"""GDN value-head sharding across ranks (one process per GPU).

The gated delta rule is independent per value head (gdn.rs:9-24): value head hv reads
q/k head hv % H_k (gdn.rs:436-441) and owns its 128x128 state, beta and decay.  So the
H_v value heads of a layer split across ranks with no exchange in the recurrence: a
rank keeps the state planes of its heads [h0, h0 + n), receives all H_k q/k heads,
its heads' v / alpha / b, and runs sqmix_gdn_decode / sqmix_gdn_prefill with
h_v_offset = h0.  The per-head outputs are gathered (all_gather) where the layer's
output projection needs all heads.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    """Value heads [start, start + count) of a GDN layer live on `rank`."""

    rank: int
    world: int
    start: int
    count: int

    def heads(self) -> range:
        return range(self.start, self.start + self.count)


def plan(h_v: int, world: int, rank: int) -> HeadShard:
    """Contiguous value-head ranges, as equal as possible (the first h_v % world ranks
    take one head more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if h_v < world:
        raise ValueError(f"{h_v} value heads cannot be split over {world} ranks")
    base, extra = divmod(h_v, world)
    start = rank * base + min(rank, extra)
    return HeadShard(rank=rank, world=world, start=start, count=base + (1 if rank < extra else 0))


def gather_heads(out_local: torch.Tensor, h_v: int, group=None) -> torch.Tensor:
    """All-gather per-rank outputs [..., n_local][128] into [..., h_v][128] in head order
    (the leading dims must match across ranks)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    shards = [plan(h_v, world, r) for r in range(world)]
    n_max = max(s.count for s in shards)
    lead = tuple(out_local.shape[:-2])
    pad = torch.zeros(lead + (n_max, out_local.shape[-1]), dtype=out_local.dtype, device=out_local.device)
    pad[..., :out_local.shape[-2], :] = out_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    return torch.cat([p[..., :s.count, :] for p, s in zip(parts, shards)], dim=-2)
