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


# ---------------------------------------------------------------------------
# Sharded multilayer predictive-coding network (the 2^31-connection iPC
# configuration across GPUs).
# ---------------------------------------------------------------------------
_M1 = 0xBF58476D1CE4E5B9 - (1 << 64)
_M2 = 0x94D049BB133111EB - (1 << 64)
_GOLD = 0x9E3779B97F4A7C15 - (1 << 64)


def _srl(x, k):
    """Logical right shift of int64 tensors holding uint64 bit patterns."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def mix64(x):
    """SplitMix64 finaliser on int64 tensors (uint64 bit patterns; products
    wrap modulo 2^64)."""
    x = x + _GOLD
    x = (x ^ _srl(x, 30)) * _M1
    x = (x ^ _srl(x, 27)) * _M2
    return x ^ _srl(x, 31)


def ipc_block_edges(l: int, size: int, fan_in: int, seed: int, device, row_lo: int = 0,
                    row_hi=None):
    """Connections of block l (into layer l + 1) of the multilayer network,
    destination rows [row_lo, row_hi) of that layer, destination-major: row d
    has fan_in sources in layer l chosen by a counter-based hash of (seed, l,
    d, j), weights N(0, 1/fan_in) by Box-Muller on two more hash words. Every
    rank can regenerate any part of the network without communication.
    Returns (from_id, to_id, weight) with absolute unit ids (layer l starts
    at l * size)."""
    import math

    import torch

    row_hi = size if row_hi is None else row_hi
    e = torch.arange(row_lo * fan_in, row_hi * fan_in, dtype=torch.int64, device=device)
    key = mix64(torch.full((1,), seed * 1000003 + l, dtype=torch.int64, device=device))
    h = mix64(e + key)
    src = (((h & 0xFFFFFFFF) * size) >> 32) + l * size
    u1 = (_srl(h, 32).to(torch.float64) + 0.5) * (1.0 / 4294967296.0)
    h2 = mix64(h)
    u2 = ((h2 & 0xFFFFFFFF).to(torch.float64) + 0.5) * (1.0 / 4294967296.0)
    w = (torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)
         * (1.0 / math.sqrt(fan_in))).to(torch.float32)
    to = torch.div(e, fan_in, rounding_mode="floor") + (l + 1) * size
    return src.to(torch.int32), to.to(torch.int32), w


def allgather_owned(t, n_layers: int, size: int, rank: int, world: int, send, recv,
                    group=None) -> None:
    """t holds n_layers layers of `size` units; rank q owns units
    [q*m, (q+1)*m) of each layer (m = size / world). Gathers every rank's
    owned slices into t (one collective: a fixed-size all-gather of the
    n_layers * m owned values, then one reordering copy)."""
    import torch
    import torch.distributed as dist

    m = size // world
    lo = rank * m
    send.view(n_layers, m).copy_(t.view(n_layers, size)[:, lo:lo + m])
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        parts = list(recv.view(world, n_layers * m).unbind(0))  # views of recv
        dist.all_gather(parts, send, group=group)
    t.view(n_layers, size).copy_(recv.view(world, n_layers, m).permute(1, 0, 2)
                                 .reshape(n_layers, size))


class ShardedPCNet:
    """The multilayer iPC network (layers of `size` units, `fan_in` random
    sources per destination) sharded by unit range: rank r owns units
    [r*m, (r+1)*m) of every layer, m = size / world -- the destination rows of
    every block in destination-major chunked layout, and the source rows of
    every hidden layer in source-major chunked layout (built from the whole
    block, keeping the connections whose source is owned). Per inference
    iteration two all-gathers cross GPUs: f(x) of every layer before the
    forward sweep and eps before the backward sweep (5 layers x size floats
    each); the weight update all-gathers f(x) once more. Each copy of a
    weight is updated by its owner with the same rule and inputs, so the
    copies stay bit-identical, and every row is folded over the same segments
    as on one GPU: results equal the single-GPU network's bit for bit."""

    def __init__(self, ctx, size: int, fan_in: int, n_layers: int, rank: int, world: int,
                 seed: int, *, gamma: float = 0.1, alpha: float = 0.005, group=None):
        import torch

        from . import _abi
        from .runtime import ChunkedRows

        if size % world:
            raise ValueError("size must be divisible by the number of ranks")
        self.ctx, self.size, self.L = ctx, size, n_layers
        self.rank, self.world, self.group = rank, world, group
        self.m = size // world
        self.lo = rank * self.m
        self.gamma, self.alpha = float(gamma), float(alpha)
        dev = ctx.device
        self.begin = [l * size for l in range(n_layers + 1)]
        self.fwd, self.bwd = [], {}
        for l in range(n_layers - 1):
            f, t, w = ipc_block_edges(l, size, fan_in, seed, dev)
            a, b = self.lo * fan_in, (self.lo + self.m) * fan_in
            self.fwd.append(ChunkedRows(ctx, f[a:b], t[a:b], w[a:b], self.begin[l], size,
                                        self.begin[l + 1] + self.lo, self.m))
            if l >= 1:
                self.bwd[l] = ChunkedRows(ctx, t, f, w, self.begin[l + 1], size,
                                          self.begin[l] + self.lo, self.m)
            del f, t, w
        n_units = self.begin[-1]
        self.x = torch.zeros(n_units, dtype=torch.float32, device=dev)
        self.act = torch.zeros_like(self.x)
        self.err = torch.zeros_like(self.x)
        self.bu = torch.zeros_like(self.x)
        self._send = torch.empty(n_layers * self.m, dtype=torch.float32, device=dev)
        self._recv = torch.empty(world * n_layers * self.m, dtype=torch.float32, device=dev)
        self._abi = _abi

    def own(self, t, l):
        """This rank's slice of layer l of a unit-sized tensor."""
        s = self.begin[l] + self.lo
        return t[s:s + self.m]

    def layer(self, t, l):
        return t[self.begin[l]:self.begin[l + 1]]

    def allgather_layers(self, t) -> None:
        """Every rank's owned slices of every layer -> the full vector."""
        allgather_owned(t, self.L, self.size, self.rank, self.world, self._send, self._recv,
                        self.group)

    def clamp(self, inputs, targets) -> None:
        """Clamps inputs and output targets (full vectors on every rank) and
        runs the pre-step for the owned hidden units."""
        from .runtime import _ptr, call

        self.layer(self.x, 0).copy_(inputs)
        self.layer(self.act, 0).copy_(inputs)
        self.layer(self.x, self.L - 1).copy_(targets)
        for l in range(1, self.L - 1):
            call("plx_ipc_value_update", self.ctx.handle, self.m, _ptr(self.own(self.x, l)),
                 None, None, 0.0, _ptr(self.own(self.act, l)), 0)

    def iteration(self) -> None:
        A = self._abi
        self.allgather_layers(self.act)
        for l, ch in enumerate(self.fwd):
            ch.fold(self.layer(self.act, l), self.own(self.err, l + 1), A.APPLY_IPC_ERROR,
                    value=self.own(self.x, l + 1))
        self.allgather_layers(self.err)
        # backward folds with the value-node update of the owned hidden
        # units in their epilogue (every hidden layer has one backward block)
        for l, ch in self.bwd.items():
            ch.fold_ipc_value(self.layer(self.err, l + 1), self.own(self.x, l),
                              self.own(self.err, l), self.own(self.act, l), self.gamma)

    def update(self) -> None:
        A = self._abi
        self.allgather_layers(self.act)
        for l, ch in enumerate(self.fwd):
            ch.update(self.layer(self.act, l), self.own(self.err, l + 1), A.UPDATE_HEBBIAN,
                      self.alpha)
        for l, ch in self.bwd.items():
            ch.update(self.layer(self.err, l + 1), self.own(self.act, l), A.UPDATE_HEBBIAN_T,
                      self.alpha)


# ---------------------------------------------------------------------------
# Hand-off over peer memory (one process per GPU): an all-gather buffer that
# every rank's sweep writes into directly over NVLink.
# ---------------------------------------------------------------------------
class PeerGather:
    """All-gather buffers over peer memory, double-buffered by epoch.

    Every rank holds two buffers of n_total floats, mapped into every other
    rank through CUDA IPC, and a flag array for plx_peer_barrier. Epoch k
    (counted from 1) hands off into buffer k & 1: a producer passes
    ``out_for_next()`` (all ranks' buffers of the next epoch) to
    plx_sweep_forward_hebbian_gather with its slice offset and
    ``n_total`` as the buffer length, then calls ``barrier()``, after which
    every rank's slice of that epoch has landed in every buffer and
    ``gathered_ptr()`` / ``copy_to()`` read it.

    Why two buffers: a rank that has passed barrier k may start the sweep of
    epoch k + 1 and store into the other ranks' buffers while a slower rank
    is still reading epoch k (a copy, or a next layer gathering from it).
    Those stores go to the other buffer. They can only come back to epoch
    k's buffer at epoch k + 2, which needs every rank's barrier k + 1, and
    each rank's barrier is queued on its stream after its own reads of
    epoch k. The contract for consumers: enqueue every read of epoch k's
    buffer on the context's stream before the barrier of epoch k + 1."""

    def __init__(self, ctx, n_total: int, rank: int, world: int, group=None):
        import ctypes
        from ctypes import c_void_p

        import torch.distributed as dist

        from . import _abi
        from .runtime import call

        if world > _abi.MAX_PEERS:
            raise ValueError(f"at most {_abi.MAX_PEERS} ranks")
        self.ctx, self.rank, self.world, self.n_total = ctx, rank, world, n_total
        self._own = []
        handles = []
        for nbytes in (4 * n_total, 4 * n_total, 8 * world):
            ptr = c_void_p()
            h = ctypes.create_string_buffer(_abi.IPC_HANDLE_BYTES)
            call("plx_peer_alloc", ctx.handle, nbytes, ctypes.byref(ptr), h)
            self._own.append(ptr.value)
            handles.append(h.raw)
        everyone = [None] * world
        dist.all_gather_object(everyone, handles, group=group)
        self._opened = []
        bufs, flags = ([], []), []
        for q in range(world):
            if q == rank:
                got = self._own
            else:
                got = []
                for h in everyone[q]:
                    ptr = c_void_p()
                    call("plx_peer_open", ctx.handle, ctypes.create_string_buffer(h, len(h)),
                         ctypes.byref(ptr))
                    self._opened.append(ptr.value)
                    got.append(ptr.value)
            bufs[0].append(got[0])
            bufs[1].append(got[1])
            flags.append(got[2])
        self._peer_out = tuple((c_void_p * world)(*b) for b in bufs)
        self.flags = (c_void_p * world)(*flags)
        self._local = (self._own[0], self._own[1])
        self.epoch = 0

    @property
    def peer_out(self):
        """Every rank's buffer of the next epoch (what the sweep stores into)."""
        return self._peer_out[(self.epoch + 1) & 1]

    def out_for_next(self):
        return self.peer_out

    def gathered_ptr(self) -> int:
        """This rank's buffer of the last completed epoch (device address)."""
        if self.epoch == 0:
            raise RuntimeError("no hand-off has completed yet")
        return self._local[self.epoch & 1]

    def gathered(self):
        """This rank's buffer of the last completed epoch as a float32 CUDA
        tensor (a view, no copy). It holds that epoch's values until the
        barrier of epoch + 2: read it (e.g. as the next sweep's sources) on
        the context's stream before the next barrier."""
        import torch

        class _View:  # zero-copy export of the peer-memory buffer to torch
            __cuda_array_interface__ = {"shape": (self.n_total,), "typestr": "<f4",
                                        "data": (self.gathered_ptr(), False), "version": 3,
                                        "strides": None}

        return torch.as_tensor(_View(), device=self.ctx.device)

    def barrier(self) -> None:
        from .runtime import call

        self.epoch += 1
        call("plx_peer_barrier", self.ctx.handle, self.flags, self.world, self.rank,
             self.epoch)

    def copy_to(self, out) -> None:
        """Copies this rank's buffer of the last completed epoch into a
        float32 CUDA tensor (on the context's stream)."""
        from .runtime import _ptr, call

        call("plx_copy_device", self.ctx.handle, _ptr(out), self.gathered_ptr(),
             4 * self.n_total)

    def close(self) -> None:
        from .runtime import call

        for p in self._opened:
            call("plx_peer_close", self.ctx.handle, p)
        for p in self._own:
            call("plx_peer_free", self.ctx.handle, p)
        self._opened, self._own = [], []
