"""Row-window sharding across the GPUs of one box.

Windows are independent and write disjoint output rows, so the path shards
with no data-path collective: rank r owns a contiguous window range
[lo_r, hi_r) cut at equal cost prefix sums, holds the Q / O rows of that
range (its slab) and a replica of K and V.  The only collective is the
optional all-gather of O, for callers that need the full output on every
rank.

Cost of a window = its active blocks + WINDOW_COST: every block moves a K and
a V tile (64*d bytes per head), every window reads a Q tile and writes an O
tile (32*d + 64*d bytes per head), i.e. 1.5 blocks' worth.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

WINDOW_COST = 1.5


def partition_windows(window_offsets, world_size: int, window_cost: float = WINDOW_COST) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) window ranges, one per rank, of near-equal cost."""
    off = np.asarray(window_offsets, dtype=np.int64)
    nrw = off.shape[0] - 1
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    cost = np.diff(off).astype(np.float64) + window_cost
    prefix = np.concatenate([[0.0], np.cumsum(cost)])
    total = prefix[-1]
    cuts = [0]
    for r in range(1, world_size):
        c = int(np.searchsorted(prefix, total * r / world_size, side="left"))
        cuts.append(min(max(c, cuts[-1]), nrw))
    cuts.append(nrw)
    return [(cuts[r], cuts[r + 1]) for r in range(world_size)]


def slab_rows(lo: int, hi: int, num_nodes: int) -> Tuple[int, int]:
    """Node rows [r0, r1) covered by windows [lo, hi)."""
    return min(16 * lo, num_nodes), min(16 * hi, num_nodes)


def rank_order(global_order, lo: int, hi: int):
    """The global balanced order restricted to [lo, hi), order preserved
    (still descending by block count).  Works on numpy arrays and torch
    tensors alike."""
    keep = (global_order >= lo) & (global_order < hi)
    return global_order[keep]


def gather_rows(slab, slabs: Sequence[Tuple[int, int]], group=None):
    """All-gather per-rank row slabs (torch tensors, first dim = rows) into
    the full tensor on every rank.  Slabs may differ in size: each rank pads
    to the largest slab, one all_gather moves them, and the padding is
    dropped.  Every rank makes the same collective call."""
    import torch
    import torch.distributed as dist

    sizes = [r1 - r0 for r0, r1 in slabs]
    m = max(sizes) if sizes else 0
    if slab.shape[0] != sizes[dist.get_rank(group)]:
        raise ValueError("slab rows disagree with the partition")
    padded = torch.zeros((m,) + tuple(slab.shape[1:]), dtype=slab.dtype, device=slab.device)
    padded[: slab.shape[0]] = slab
    bufs = [torch.empty_like(padded) for _ in sizes]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([b[:s] for b, s in zip(bufs, sizes)], dim=0)
