"""Destination-range sharding of a layer over one process per GPU.

A layer's connections are sorted by ToId, so a contiguous range of
destination rows owns a contiguous range of connections: each rank keeps the
connections of its rows, a replica of the source activations, and writes only
its rows' activations. After every sweep the ranks all-gather their
destination slices (the hand-off to the next layer); nothing else crosses
GPUs. Rows are cut so that every rank holds about the same number of
connections (the sweep is bound by connection bytes, not rows).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


@dataclass(frozen=True)
class Shard:
    rank: int
    row_lo: int   # first destination row (relative to the layer's rows)
    row_hi: int   # one past the last
    edge_lo: int  # first connection
    edge_hi: int  # one past the last

    @property
    def n_rows(self) -> int:
        return self.row_hi - self.row_lo

    @property
    def n_edges(self) -> int:
        return self.edge_hi - self.edge_lo


def balanced_shards(row_ptr: Sequence[int], world: int) -> List[Shard]:
    """Contiguous row ranges with about n_edges / world connections each.

    row_ptr: n_rows + 1 non-decreasing offsets (CSR over dst-sorted
    connections). Cut k is the first row whose start offset is at least
    k * n_edges / world, so shards differ by at most one row's connections
    from the even split. Every rank gets a (possibly empty) range."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    if rp.ndim != 1 or rp.size < 1:
        raise ValueError("row_ptr must hold n_rows + 1 offsets")
    if world < 1:
        raise ValueError("world must be >= 1")
    if np.any(np.diff(rp) < 0):
        raise ValueError("row_ptr must be non-decreasing")
    n_rows, n_edges = rp.size - 1, int(rp[-1])
    cuts = [0]
    for k in range(1, world):
        target = (k * n_edges) // world
        cuts.append(max(cuts[-1], int(np.searchsorted(rp[:-1], target, side="left"))))
    cuts.append(n_rows)
    return [Shard(r, cuts[r], cuts[r + 1], int(rp[cuts[r]]), int(rp[cuts[r + 1]]))
            for r in range(world)]


def even_shards(n_rows: int, world: int, row_ptr: Sequence[int] | None = None) -> List[Shard]:
    """Equal row counts (n_rows divisible by world): the layout the
    fixed-size all-gather needs without padding."""
    if n_rows % world:
        raise ValueError("n_rows must be divisible by world for even shards")
    per = n_rows // world
    rp = None if row_ptr is None else np.asarray(row_ptr, dtype=np.int64)
    out = []
    for r in range(world):
        lo, hi = r * per, (r + 1) * per
        e_lo = int(rp[lo]) if rp is not None else 0
        e_hi = int(rp[hi]) if rp is not None else 0
        out.append(Shard(r, lo, hi, e_lo, e_hi))
    return out


def allgather_rows(local, shards: Sequence[Shard], group=None):
    """All-gathers every rank's destination slice into the full row vector
    (torch tensors; NCCL or gloo). Slices are padded to the largest shard so
    one fixed-size collective serves uneven shards; the result drops the
    padding and follows row order."""
    import torch
    import torch.distributed as dist

    world = len(shards)
    width = max(s.n_rows for s in shards)
    buf = torch.zeros(width, dtype=local.dtype, device=local.device)
    buf[:local.numel()].copy_(local)
    if dist.get_backend(group) == "nccl":
        out = torch.empty(width * world, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, buf, group=group)
        parts = [out[r * width:r * width + shards[r].n_rows] for r in range(world)]
    else:
        got = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(got, buf, group=group)
        parts = [got[r][:shards[r].n_rows] for r in range(world)]
    return torch.cat(parts)
