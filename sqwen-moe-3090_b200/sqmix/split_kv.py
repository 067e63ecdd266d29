"""Split-KV decode across ranks (one process per GPU, long-context decode).

Each rank keeps a contiguous slice of every full-attention layer's keys in its own
KvCache, computes normalised partial attention (O_p, LSE_p) over that slice (RoPE
positions offset by the slice start), and the partials of all ranks are merged:
    out = sum_p O_p exp(LSE_p - L) * sigmoid(gate),   L = log sum_p exp(LSE_p).
This is exact: softmax over the union of disjoint key sets.  The step's new row is
appended by the rank whose slice holds its position.

PeerMerge.decode (sqmix_fa_decode_peers) does a layer in two launches: the decode and
a split merge that exchanges the partials with the other ranks through peer memory
over NVLink.  gather() + attn_merge_lse is the collective-library route (NCCL over
NVLink, gloo on the host in the CPU tests).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import SQMIX_FA_OVERLAP_PREV, PeerMergeArgs, check, lib
from .ops import KV_PAD, _fa_args, _ptr, _stream, new_fa_workspace

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


class PeerMerge:
    """The (O, LSE) exchange of split-KV decode over peer memory (NVLink P2P): one
    peer buffer per rank, IPC handles swapped through the process group, and one
    sqmix_attn_merge_peers launch per layer that publishes this rank's partial and
    merges everyone's.  Replaces gather() + attn_merge_lse with a single kernel.

    n_slots: merges per step (one per layer).  Every rank calls merge() for the same
    slots in the same order.  close() after the last step (all ranks)."""

    IPC_BYTES = 64

    def __init__(self, n_slots: int, rows: int = 16, group=None, device=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_slots = int(n_slots)
        self.rows = int(rows)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(self.IPC_BYTES)
        check(lib().sqmix_peer_buffer_create(self.n_slots, ctypes.byref(own), handle), "peer_buffer_create")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            check(lib().sqmix_peer_buffer_open(ctypes.create_string_buffer(h, self.IPC_BYTES), ctypes.byref(p)),
                  "peer_buffer_open")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def merge(self, o_local: torch.Tensor, lse_local: torch.Tensor, slot: int, gate: torch.Tensor | None = None,
              out: torch.Tensor | None = None, lse_out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """o_local [rows][256] f32 and lse_local [rows] (natural log) of this rank's key
        slice -> out [rows][256] over all ranks (* sigmoid(gate) when given)."""
        o_local = o_local.reshape(self.rows, 256)
        lse_local = lse_local.reshape(self.rows)
        if out is None:
            out = torch.empty((self.rows, 256), dtype=torch.float32, device=o_local.device)
        if gate is not None:
            gate = gate.reshape(self.rows, 256)
            if gate.dtype != torch.float32 or not gate.is_contiguous():
                gate = gate.float().contiguous()
        a = PeerMergeArgs(n_ranks=self.world, rank=self.rank, slot=int(slot), n_slots=self.n_slots, rows=self.rows,
                          buffers=_ptr(self.ptrs), o_local=_ptr(o_local), lse_local=_ptr(lse_local), gate=_ptr(gate),
                          out=_ptr(out), lse_out=_ptr(lse_out), status=_ptr(self.status))
        check(lib().sqmix_attn_merge_peers(ctypes.byref(a), _stream(stream)), "attn_merge_peers")
        return out

    def decode(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, capacity: int,
               n_kv: torch.Tensor, q_pos0: torch.Tensor, slot: int, gate: torch.Tensor | None = None,
               out: torch.Tensor | None = None, lse: torch.Tensor | None = None, scale: float = 1.0 / 16.0,
               rope_n_rot: int = 0, rope_freq_base: float = 1e7, rope_pos_offset: int = 0,
               workspace: torch.Tensor | None = None, n_splits: int = 0, config: int = 0,
               k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None, overlap_prev: bool = False,
               stream=None) -> torch.Tensor:
        """One layer of split-KV decode (sqmix_fa_decode_peers): attention of q [n_q][16][256]
        over this rank's key slice (n_kv, q_pos0 in slice rows; rope_pos_offset = the slice
        start), the exchange with every other rank and the merged, gated output over all
        ranks' keys in `out` [n_q][16][256] (and the merged LSE in `lse`).  Arguments as for
        flash_attn_ext; the rank owning the step's rows passes k_new / v_new."""
        if workspace is None:
            workspace = new_fa_workspace(q.shape[0], n_splits, q.device)
        a, out = _fa_args(q, k_cache, v_cache, capacity, n_kv, q_pos0, gate, scale, rope_n_rot, rope_freq_base,
                          rope_pos_offset, out, lse, workspace, n_splits, config, k_new, v_new,
                          SQMIX_FA_OVERLAP_PREV if overlap_prev else 0)
        pm = PeerMergeArgs(n_ranks=self.world, rank=self.rank, slot=int(slot), n_slots=self.n_slots,
                           rows=16 * a.n_q, buffers=_ptr(self.ptrs), status=_ptr(self.status))
        check(lib().sqmix_fa_decode_peers(ctypes.byref(a), ctypes.byref(pm), _stream(stream)), "fa_decode_peers")
        return out

    def reset(self, stream=None) -> None:
        """Zero this rank's buffer and status (every rank, after all have stopped calling):
        the way back to a consistent state after a wait gave up."""
        check(lib().sqmix_peer_buffer_reset(ctypes.c_void_p(self._own), self.n_slots, _stream(stream)),
              "peer_buffer_reset")
        self.status.zero_()

    def ok(self) -> bool:
        """False if a bounded wait for a peer gave up (synchronises)."""
        return int(self.status.item()) == 0

    def close(self):
        """Unmap the peers and free this rank's buffer, after every rank is done."""
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            check(lib().sqmix_peer_buffer_close(ctypes.c_void_p(p)), "peer_buffer_close")
        self._opened = []
        dist.barrier(group=self.group)
        check(lib().sqmix_peer_buffer_destroy(ctypes.c_void_p(self._own)), "peer_buffer_destroy")
        self._own = None
