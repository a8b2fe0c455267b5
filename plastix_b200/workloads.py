"""Seeded synthetic workloads (no public dataset exists for this path).

Each generator returns the reference's SoA field arrays for one network
shape, as numpy arrays (small, CPU-checkable cases) or torch tensors built on
the device (benchmark sizes). Distributions follow the workload definitions:

* single sparse layer: ``n_src`` inputs, ``n_dst`` destinations, ``n_edges``
  uniform random (src, dst) pairs, stable-sorted by dst; weights
  N(0, 0.05^2); input activations U(0, 1); traces 0.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class SparseLayer:
    n_src: int
    n_dst: int
    from_id: np.ndarray  # u32, absolute unit ids in [0, n_src)
    to_id: np.ndarray    # u32, absolute unit ids in [n_src, n_src + n_dst), sorted
    weight: np.ndarray   # f32
    trace: np.ndarray    # f32
    act_in: np.ndarray   # f32, n_src


def sparse_layer(n_src: int, n_dst: int, n_edges: int, seed: int = 0,
                 w_std: float = 0.05) -> SparseLayer:
    rng = np.random.default_rng(seed)
    src = rng.integers(0, n_src, n_edges, dtype=np.uint32)
    dst = rng.integers(0, n_dst, n_edges, dtype=np.uint32)
    order = np.argsort(dst, kind="stable")
    src = np.ascontiguousarray(src[order])
    to = np.ascontiguousarray(dst[order] + np.uint32(n_src))
    w = rng.normal(0.0, w_std, n_edges).astype(np.float32)
    act = rng.random(n_src, dtype=np.float32)
    return SparseLayer(n_src, n_dst, src, to, w, np.zeros(n_edges, np.float32), act)


def sparse_layer_rows(n_src: int, row_lengths, seed: int = 0, w_std: float = 0.05
                      ) -> SparseLayer:
    """A layer with an explicit length per destination row (edge cases:
    empty rows, long rows, rows crossing tile boundaries)."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(row_lengths, dtype=np.int64)
    n_dst = lens.size
    n = int(lens.sum())
    to = np.repeat(np.arange(n_dst, dtype=np.uint32), lens) + np.uint32(n_src)
    src = rng.integers(0, n_src, n, dtype=np.uint32)
    w = rng.normal(0.0, w_std, n).astype(np.float32)
    act = rng.random(n_src, dtype=np.float32)
    return SparseLayer(n_src, n_dst, src, np.ascontiguousarray(to), w,
                       np.zeros(n, np.float32), act)


def sparse_layer_device(n_src: int, n_dst: int, n_edges: int, seed: int, device,
                        w_std: float = 0.05):
    """Benchmark-size version generated on the device with torch's seeded
    generator: (from_id i32, to_id i32 sorted, weight f32, act_in f32)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    src = torch.randint(0, n_src, (n_edges,), generator=g, device=device, dtype=torch.int64)
    dst = torch.randint(0, n_dst, (n_edges,), generator=g, device=device, dtype=torch.int64)
    dst_sorted, order = torch.sort(dst, stable=True)
    from_id = src[order].to(torch.int32)
    del src, order
    to_id = (dst_sorted + n_src).to(torch.int32)
    del dst, dst_sorted
    w = torch.randn(n_edges, generator=g, device=device, dtype=torch.float32) * w_std
    act = torch.rand(n_src, generator=g, device=device, dtype=torch.float32)
    return from_id, to_id, w, act


def level_graph(n_units: int, n_input: int, n_conns: int, seed: int = 0, *,
                back_edges: int = 0, dead_frac: float = 0.0, into_inputs: int = 0):
    """Connections for level tests (RecomputeLevels): each connection runs
    from a lower to a higher unit id, so the graph is acyclic, except
    `back_edges` from higher to lower non-input ids (cycles) and `into_inputs`
    from non-input units into input units. Returns (from_id, to_id, dead);
    dead is None unless dead_frac > 0."""
    rng = np.random.default_rng(seed)
    n_dag = n_conns - back_edges - into_inputs
    to = rng.integers(max(n_input, 1), n_units, n_dag).astype(np.int64)
    frm = (rng.random(n_dag) * to).astype(np.int64)  # uniform in [0, to)
    parts_f, parts_t = [frm], [to]
    if back_edges:
        a = rng.integers(n_input, n_units, back_edges)
        b = rng.integers(n_input, n_units, back_edges)
        parts_f.append(np.maximum(a, b))
        parts_t.append(np.minimum(a, b))
    if into_inputs:
        parts_f.append(rng.integers(n_input, n_units, into_inputs))
        parts_t.append(rng.integers(0, max(n_input, 1), into_inputs))
    frm = np.concatenate(parts_f).astype(np.uint32)
    to = np.concatenate(parts_t).astype(np.uint32)
    order = rng.permutation(frm.size)
    frm, to = np.ascontiguousarray(frm[order]), np.ascontiguousarray(to[order])
    dead = None
    if dead_frac > 0:
        dead = (rng.random(frm.size) < dead_frac).astype(np.uint8)
    return frm, to, dead
