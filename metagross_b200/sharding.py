"""Sequence sharding over the GPUs of one node.

Decode attention over a paged cache has no cross-sequence reduction, so a
batch is split by sequence: each rank owns its sequences' pages, allocator,
block tables and decode plan, and runs append + attention with no
communication; once per step the last layer's outputs are gathered (NCCL
all-gather over NVLink) back into the global sequence order.

``lpt_shard`` balances the ranks by context length with the greedy
longest-processing-time rule: sequences in decreasing length order, each to
the rank with the least total length so far (ties to the lower rank, equal
lengths in index order), so every rank sees the same deterministic split.
"""
from __future__ import annotations

import numpy as np
import torch


def lpt_shard(lens, world: int, equal_counts: bool = False):
    """Partition sequence indices over ``world`` ranks by total length.

    Returns a list of ``world`` int64 arrays (ascending indices per rank).
    The largest rank load is at most (4/3 - 1/(3*world)) of the optimum.
    ``equal_counts``: every rank also gets ceil or floor(N / world) sequences
    (the first N % world ranks one more), so the ranks' output blocks have
    one size and an all-gather needs no padding copy; the greedy step then
    picks the least-loaded rank that still has room."""
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    lens = np.asarray(lens, dtype=np.int64)
    if lens.ndim != 1:
        raise ValueError("lens must be 1-D")
    if (lens < 0).any():
        raise ValueError("lengths must be non-negative")
    order = np.lexsort((np.arange(lens.size), -lens))  # longest first, index order within ties
    load = np.zeros(world, dtype=np.int64)
    room = np.full(world, np.iinfo(np.int64).max, dtype=np.int64)
    if equal_counts:
        room = np.full(world, lens.size // world, dtype=np.int64)
        room[: lens.size % world] += 1
    owner = np.empty(lens.size, dtype=np.int64)
    big = np.iinfo(np.int64).max
    for i in order:
        r = int(np.argmin(np.where(room > 0, load, big)))  # first minimum among ranks with room
        owner[i] = r
        load[r] += lens[i]
        room[r] -= 1
    return [np.flatnonzero(owner == r) for r in range(world)]


def shard_loads(lens, shards):
    lens = np.asarray(lens, dtype=np.int64)
    return [int(lens[s].sum()) for s in shards]


class ShardGather:
    """Gathers per-rank outputs ``[n_r, ...]`` into the global order ``[N, ...]``
    with one all_gather_into_tensor of equal-size (padded) blocks.

    ``shards`` is the same list on every rank (from ``lpt_shard``)."""

    def __init__(self, shards, rank: int, feature_shape, dtype, device):
        self.shards = [np.asarray(s, dtype=np.int64) for s in shards]
        self.world = len(self.shards)
        self.rank = rank
        self.n_max = max((s.size for s in self.shards), default=0)
        self.n = int(sum(s.size for s in self.shards))
        self.send = torch.zeros((self.n_max, *feature_shape), dtype=dtype, device=device)
        self.recv = torch.zeros((self.world * self.n_max, *feature_shape), dtype=dtype, device=device)
        # position in the padded receive buffer of every global sequence
        src = np.empty(self.n, dtype=np.int64)
        for r, s in enumerate(self.shards):
            src[s] = r * self.n_max + np.arange(s.size)
        self.src = torch.as_tensor(src, device=device)

    def __call__(self, local_out: torch.Tensor, group=None, reorder: bool = True) -> torch.Tensor:
        """All ranks' outputs.  reorder=True: [N, ...] in global sequence order.
        reorder=False: the padded [world * n_max, ...] rank-major buffer itself
        (rank r's sequences shards[r] at rows r * n_max ...; ``lengths`` gives
        each rank's count), with no reordering pass.  A local block that
        already has n_max contiguous rows is sent as it is, without a copy."""
        import torch.distributed as dist

        n_r = self.shards[self.rank].size
        if local_out.shape[0] != n_r:
            raise ValueError(f"rank {self.rank} owns {n_r} sequences, got {local_out.shape[0]} outputs")
        if n_r == self.n_max and local_out.is_contiguous() and local_out.dtype == self.send.dtype:
            send = local_out
        else:
            self.send[:n_r].copy_(local_out)
            send = self.send
        dist.all_gather_into_tensor(self.recv, send, group=group)
        return self.recv.index_select(0, self.src) if reorder else self.recv

    @property
    def lengths(self):
        """Sequences per rank (the valid rows of each n_max block of the padded buffer)."""
        return [int(s.size) for s in self.shards]
