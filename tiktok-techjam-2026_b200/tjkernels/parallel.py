"""Batch sharding across GPUs (one process per GPU).

Every layer of the encoder works within one sequence (row-wise GEMMs and
LayerNorms, causal self-attention inside a sequence), so sequences are
independent: a batch splits across ranks with no collective in the forward.
Weights are replicated.  ``shard_range`` gives each rank a contiguous slice of
the batch; ``balanced_shards`` instead balances the valid-token work when
padded tiles are skipped.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple


def shard_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) of sequences for ``rank``; sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def balanced_shards(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Assign sequences to ranks so each rank's sum of causal work
    (len*(len+1)/2 attention plus len for the GEMMs) is balanced: greedy
    longest-first onto the least-loaded rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: -int(lengths[i]))
    loads = [0.0] * world
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        n = int(lengths[i])
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += n * (n + 1) / 2 + n
    return [sorted(s) for s in shards]


def balanced_equal_shards(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Like ``balanced_shards`` but every rank gets the same number of
    sequences (``len(lengths)`` must be a multiple of ``world``): sort by
    causal work, longest first, and deal in snake order (0..w-1, w-1..0, ...),
    so each rank's batch has the same shape and close to the same work."""
    if world <= 0 or len(lengths) % world != 0:
        raise ValueError("the number of sequences must be a positive multiple of world")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    shards: List[List[int]] = [[] for _ in range(world)]
    for k, i in enumerate(order):
        rnd, pos = divmod(k, world)
        shards[pos if rnd % 2 == 0 else world - 1 - pos].append(i)
    return [sorted(s) for s in shards]
