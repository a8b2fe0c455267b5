"""Host-side plumbing over the C ABI: device context, dst-sorted CSR index,
and the sweep entry points on torch tensors (device memory and streams come
from PyTorch; every computation runs in libplastix_b200.so).

Connection and unit fields are the reference's SoA arrays
(include/plastix/conn.hpp:31-36, include/plastix/unit_state.hpp:38-44), one
tensor per field. u32 fields (FromId, ToId) are stored as int32 tensors with
the same bit pattern.
"""
from __future__ import annotations

from ctypes import byref, c_void_p
from typing import Optional

import torch

from . import _abi
from ._abi import Chunked, Csr, Field, Sliced, call


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


class Context:
    """One device + the stream kernels are enqueued on (torch's current
    stream of that device unless given)."""

    def __init__(self, device: int = 0, stream: Optional[torch.cuda.Stream] = None):
        self.device = torch.device("cuda", device)
        self._stream = stream or torch.cuda.current_stream(self.device)
        h = c_void_p()
        call("plx_ctx_create", device, c_void_p(self._stream.cuda_stream), byref(h))
        self.handle = h

    @property
    def stream(self) -> torch.cuda.Stream:
        return self._stream

    def use_stream(self, stream: torch.cuda.Stream) -> None:
        self._stream = stream
        call("plx_ctx_set_stream", self.handle, c_void_p(stream.cuda_stream))

    def set_timeout_ns(self, ns: int) -> None:
        call("plx_ctx_set_timeout_ns", self.handle, ns)

    def sync(self) -> None:
        """Waits for the stream and raises if a kernel reported an error."""
        call("plx_ctx_sync", self.handle)

    def close(self) -> None:
        if self.handle:
            _abi.lib().plx_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DstCsr:
    """CSR index over connections sorted by ToId: rows are the destination
    units [row_base, row_base + n_rows)."""

    def __init__(self, ctx: Context, to_id: torch.Tensor, row_base: int, n_rows: int,
                 *, use_to_id: bool = True):
        n_edges = int(to_id.numel())
        self.row_ptr = torch.empty(n_rows + 1, dtype=torch.int32, device=ctx.device)
        call("plx_csr_row_ptr", ctx.handle, c_void_p(_ptr(to_id) if n_edges else None),
             n_edges, row_base, n_rows, c_void_p(_ptr(self.row_ptr)))
        self._init_plan(ctx, n_edges, n_rows)
        self.set_to_id(to_id if use_to_id else None, row_base)

    def set_to_id(self, to_id: Optional[torch.Tensor], row_base: int) -> None:
        """Enables the warp fast path (needs the dst-sorted ToId field)."""
        self.to_id = to_id
        self.struct.to_id = _ptr(to_id) if to_id is not None and to_id.numel() else None
        self.struct.row_base = row_base

    @classmethod
    def from_sorted_async(cls, ctx: Context, to_id: torch.Tensor, row_base: int,
                          n_rows: int, row_ptr: Optional[torch.Tensor] = None,
                          plan: Optional[torch.Tensor] = None) -> "DstCsr":
        """Builds row_ptr and the plan without a host synchronisation (row
        counts stay unknown; the sweeps read them on the device). Reuses the
        given buffers when they are large enough."""
        self = cls.__new__(cls)
        n_edges = int(to_id.numel())
        if row_ptr is None or row_ptr.numel() < n_rows + 1:
            row_ptr = torch.empty(n_rows + 1, dtype=torch.int32, device=ctx.device)
        self.row_ptr = row_ptr
        call("plx_csr_row_ptr", ctx.handle, c_void_p(_ptr(to_id) if n_edges else None),
             n_edges, row_base, n_rows, c_void_p(_ptr(self.row_ptr)))
        words = _abi.lib().plx_csr_plan_words(n_edges, n_rows)
        if plan is None or plan.numel() < words:
            plan = torch.empty(int(words), dtype=torch.int32, device=ctx.device)
        self.plan = plan
        self.struct = Csr()
        call("plx_csr_plan_async", ctx.handle, c_void_p(_ptr(self.row_ptr)), n_rows, n_edges,
             c_void_p(_ptr(self.plan)), words, byref(self.struct))
        self.n_edges, self.n_rows = n_edges, n_rows
        self.n_wide = self.n_long = self.n_short = _abi.COUNT_UNKNOWN
        self.set_to_id(to_id, row_base)
        return self

    @classmethod
    def from_row_ptr(cls, ctx: Context, row_ptr: torch.Tensor) -> "DstCsr":
        self = cls.__new__(cls)
        self.row_ptr = row_ptr.to(device=ctx.device, dtype=torch.int32).contiguous()
        n_rows = int(self.row_ptr.numel()) - 1
        n_edges = int(self.row_ptr[-1].item())
        self._init_plan(ctx, n_edges, n_rows)
        self.set_to_id(None, 0)
        return self

    def _init_plan(self, ctx: Context, n_edges: int, n_rows: int) -> None:
        words = _abi.lib().plx_csr_plan_words(n_edges, n_rows)
        self.plan = torch.empty(int(words), dtype=torch.int32, device=ctx.device)
        self.struct = Csr()
        call("plx_csr_plan", ctx.handle, c_void_p(_ptr(self.row_ptr)), n_rows, n_edges,
             c_void_p(_ptr(self.plan)), words, byref(self.struct))
        self.n_edges = n_edges
        self.n_rows = n_rows
        self.n_wide = self.struct.n_wide
        self.n_long = self.struct.n_long
        self.n_short = self.struct.n_short


def sweep_forward(ctx: Context, csr: DstCsr, from_id: torch.Tensor, weight: torch.Tensor,
                  act_src: torch.Tensor, act_dst: Optional[torch.Tensor] = None, *,
                  apply: int = _abi.APPLY_IDENTITY, dead: Optional[torch.Tensor] = None,
                  value: Optional[torch.Tensor] = None,
                  err_out: Optional[torch.Tensor] = None) -> None:
    call("plx_sweep_forward", ctx.handle, byref(csr.struct), _ptr(from_id), _ptr(weight),
         _ptr(dead), _ptr(act_src), int(act_src.numel()), apply, _ptr(act_dst),
         _ptr(value), _ptr(err_out))


def sweep_forward_rows(ctx: Context, row_ptr: torch.Tensor, from_id: torch.Tensor,
                       weight: torch.Tensor, act_src: torch.Tensor,
                       act_dst: Optional[torch.Tensor] = None, *,
                       apply: int = _abi.APPLY_IDENTITY, dead: Optional[torch.Tensor] = None,
                       value: Optional[torch.Tensor] = None,
                       err_out: Optional[torch.Tensor] = None) -> None:
    """``sweep_forward`` over row offsets alone: one thread per row, a left
    fold in connection order (for layers of a few connections per row)."""
    call("plx_sweep_forward_rows", ctx.handle, _ptr(row_ptr), int(row_ptr.numel()) - 1,
         _ptr(from_id), _ptr(weight), _ptr(dead), _ptr(act_src), int(act_src.numel()), apply,
         _ptr(act_dst), _ptr(value), _ptr(err_out))


def sweep_forward_hebbian(ctx: Context, csr: DstCsr, from_id: torch.Tensor,
                          act_src: torch.Tensor, w_in: torch.Tensor, w_out: torch.Tensor,
                          trace_in: torch.Tensor, trace_out: torch.Tensor,
                          act_dst: torch.Tensor, *, decay: float, rate: float,
                          dead: Optional[torch.Tensor] = None) -> None:
    call("plx_sweep_forward_hebbian", ctx.handle, byref(csr.struct), _ptr(from_id),
         _ptr(dead), _ptr(act_src), int(act_src.numel()), _ptr(w_in), _ptr(w_out),
         _ptr(trace_in), _ptr(trace_out), decay, rate, _ptr(act_dst))


def sweep_update(ctx: Context, csr: DstCsr, from_id: torch.Tensor, act_src: torch.Tensor,
                 post: torch.Tensor, w_in: torch.Tensor, w_out: torch.Tensor, *,
                 kind: int, rate: float, dead: Optional[torch.Tensor] = None) -> None:
    call("plx_sweep_update", ctx.handle, byref(csr.struct), _ptr(from_id), _ptr(dead),
         _ptr(act_src), int(act_src.numel()), _ptr(post), kind, rate, _ptr(w_in),
         _ptr(w_out))


class SlicedRows:
    """The warp-sliced row layout of a destination-sorted CSR (see
    plx_sliced_plan): rows in windows of 512, ordered by length inside a
    window and dealt 32 per slice, one row per lane; slot order for every
    connection field, with ``pack`` / ``unpack`` between reference order and
    slot order."""

    def __init__(self, ctx: Context, csr: "DstCsr"):
        dev = ctx.device
        self.ctx = ctx
        n_rows, n_edges = csr.n_rows, csr.n_edges
        lib = _abi.lib()
        n_slices = int(lib.plx_sliced_n_slices(n_rows))
        self.slice_ptr = torch.empty(n_slices + 1, dtype=torch.int64, device=dev)
        self.lane_row = torch.empty(n_slices * 32, dtype=torch.int32, device=dev)
        self.lane_len = torch.empty(n_slices * 32, dtype=torch.int32, device=dev)
        nb = int(lib.plx_sliced_plan_scratch_bytes(n_rows))
        scratch = torch.empty(nb, dtype=torch.uint8, device=dev)
        self.struct = Sliced()
        call("plx_sliced_plan", ctx.handle, _ptr(csr.row_ptr), n_rows, n_edges,
             byref(self.struct), _ptr(self.slice_ptr), _ptr(self.lane_row), _ptr(self.lane_len),
             _ptr(scratch), nb)
        del scratch
        self.n_slots = int(self.struct.n_slots)
        self.perm = torch.empty(max(self.n_slots, 4), dtype=torch.int32, device=dev)
        call("plx_sliced_perm", ctx.handle, byref(self.struct), _ptr(csr.row_ptr),
             _ptr(self.perm))
        self.n_rows, self.n_edges = n_rows, n_edges

    def pack(self, ref: torch.Tensor) -> torch.Tensor:
        """A field in slot order (padding slots zero) from reference order."""
        out = torch.zeros(max(self.n_slots, 4), dtype=ref.dtype, device=ref.device)
        if self.n_slots:
            call("plx_sliced_pack", self.ctx.handle, byref(self.struct), _ptr(ref.contiguous()),
                 _ptr(out), ref.element_size())
        return out

    def unpack(self, slot: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A field in reference order from slot order."""
        if out is None:
            out = torch.empty(self.n_edges, dtype=slot.dtype, device=slot.device)
        if self.n_slots:
            call("plx_sliced_unpack", self.ctx.handle, byref(self.struct), _ptr(slot),
                 _ptr(out), slot.element_size())
        return out


class HebbianSweepLayer:
    """One sparse layer stepped like ``Network::DoStep`` in Pipeline mode with
    the Hebbian trace rule: forward sum (identity Apply) + per-connection
    trace/weight update, fused into one pass. Arguments are in the
    reference's connection order (sorted by ToId); ``weight``/``trace``
    return the current values in that order.

    ``layout="csr"``: the connections stay in that order; weights and traces
    are double-buffered (the fused CSR sweep reads one copy and writes the
    other). ``layout="sliced"``: they are re-laid once into the warp-sliced
    row layout (SlicedRows), one lane per row, updated in place; ``weight``
    and ``trace`` then unpack to reference order on request."""

    def __init__(self, ctx: Context, n_src: int, n_dst: int, from_id: torch.Tensor,
                 to_id: torch.Tensor, weight: torch.Tensor,
                 trace: Optional[torch.Tensor] = None, *, decay: float = 0.9,
                 rate: float = 1e-3, dead: Optional[torch.Tensor] = None,
                 fast: bool = True, layout: str = "csr"):
        if layout not in ("csr", "sliced"):
            raise ValueError("layout must be 'csr' or 'sliced'")
        dev = ctx.device
        self.ctx = ctx
        self.layout = layout
        self.n_src, self.n_dst = n_src, n_dst
        self.decay, self.rate = decay, rate
        from_id = from_id.to(dev, torch.int32).contiguous()
        self.to_id = to_id.to(dev, torch.int32).contiguous()
        dead = None if dead is None else dead.to(dev, torch.uint8).contiguous()
        n = from_id.numel()
        w = weight.to(dev, torch.float32).contiguous()
        tr = torch.zeros(n, dtype=torch.float32, device=dev) if trace is None else \
            trace.to(dev, torch.float32).contiguous()
        self.csr = DstCsr(ctx, self.to_id, n_src, n_dst, use_to_id=fast)
        self.act_dst = torch.zeros(n_dst, dtype=torch.float32, device=dev)
        if layout == "sliced":
            self.slices = SlicedRows(ctx, self.csr)
            self.from_id = self.slices.pack(from_id)
            self.dead = None if dead is None else self.slices.pack(dead)
            self._w = [self.slices.pack(w)]
            self._e = [self.slices.pack(tr)]
        else:
            self.from_id, self.dead = from_id, dead
            self._w = [w.clone(), torch.empty(n, dtype=torch.float32, device=dev)]
            self._e = [tr.clone(), torch.empty(n, dtype=torch.float32, device=dev)]
        self._cur = 0

    @property
    def weight(self) -> torch.Tensor:
        if self.layout == "sliced":
            return self.slices.unpack(self._w[0])
        return self._w[self._cur]

    def _state_tensors(self):
        if self.layout == "sliced":  # slot order: a checkpoint of this layout
            return {"weight_slots": self._w[0], "trace_slots": self._e[0],
                    "act_dst": self.act_dst}
        return {"weight": self._w[self._cur], "trace": self._e[self._cur],
                "act_dst": self.act_dst}

    def save(self, path) -> None:
        """Checkpoint: current Weight and Trace, destination activations."""
        from .checkpoint import save_state
        save_state(self, path)

    def load(self, path) -> None:
        from .checkpoint import load_state
        load_state(self, path)

    @property
    def trace(self) -> torch.Tensor:
        if self.layout == "sliced":
            return self.slices.unpack(self._e[0])
        return self._e[self._cur]

    def _sliced_sweep(self, act_src, peers=None, n_peers=0, offset=0, peer_len=0):
        call("plx_sweep_forward_hebbian_sliced", self.ctx.handle, byref(self.slices.struct),
             _ptr(self.from_id), _ptr(self.dead), _ptr(act_src), int(act_src.numel()),
             _ptr(self._w[0]), _ptr(self._e[0]), self.decay, self.rate, _ptr(self.act_dst),
             peers, n_peers, offset, peer_len)

    def step(self, act_src: torch.Tensor) -> torch.Tensor:
        if self.layout == "sliced":
            self._sliced_sweep(act_src)
            return self.act_dst
        c, o = self._cur, 1 - self._cur
        sweep_forward_hebbian(self.ctx, self.csr, self.from_id, act_src, self._w[c],
                              self._w[o], self._e[c], self._e[o], self.act_dst,
                              decay=self.decay, rate=self.rate, dead=self.dead)
        self._cur = o
        return self.act_dst

    def step_gather(self, act_src: torch.Tensor, peer, offset: int) -> torch.Tensor:
        """``step`` whose destination values also land in every rank's
        all-gather buffer of the next epoch (``peer``: sharding.PeerGather)
        at ``offset``, as stores of the sweep itself; call ``peer.barrier()``
        before reading."""
        if offset < 0 or offset + self.n_dst > peer.n_total:
            raise ValueError(f"slice [{offset}, {offset + self.n_dst}) does not fit the "
                             f"hand-off buffers of {peer.n_total} floats")
        if self.layout == "sliced":
            self._sliced_sweep(act_src, peer.out_for_next(), peer.world, offset, peer.n_total)
            return self.act_dst
        c, o = self._cur, 1 - self._cur
        call("plx_sweep_forward_hebbian_gather", self.ctx.handle, byref(self.csr.struct),
             _ptr(self.from_id), _ptr(self.dead), _ptr(act_src), int(act_src.numel()),
             _ptr(self._w[c]), _ptr(self._w[o]), _ptr(self._e[c]), _ptr(self._e[o]),
             self.decay, self.rate, _ptr(self.act_dst), peer.out_for_next(), peer.world,
             offset, peer.n_total)
        self._cur = o
        return self.act_dst


# ---------------------------------------------------------------------------
# Structural change: compaction, gather, radix sort, regrowth
# ---------------------------------------------------------------------------
def _fields(pairs, flags=None):
    arr = (Field * max(1, len(pairs)))()
    for i, (src, dst) in enumerate(pairs):
        if src.dtype != dst.dtype or src.element_size() != dst.element_size():
            raise ValueError("field src/dst dtypes differ")
        arr[i] = Field(_ptr(src), _ptr(dst), src.element_size(),
                       0 if flags is None else flags[i])
    return arr


class Scratch:
    """Grow-only device scratch buffer (bytes)."""

    def __init__(self, device):
        self.device = device
        self.buf = torch.empty(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)
        return self.buf


def compact(ctx: Context, n: int, keep_kind: int, keep_src: torch.Tensor, pairs,
            count_out: torch.Tensor, *, threshold: float = 0.0, flags=None,
            perm_out: Optional[torch.Tensor] = None, scratch: Optional[Scratch] = None):
    nbytes = _abi.lib().plx_compact_scratch_bytes(n)
    s = (scratch or Scratch(ctx.device)).get(nbytes)
    f = _fields(pairs, flags)
    call("plx_compact", ctx.handle, n, keep_kind, _ptr(keep_src), threshold, f, len(pairs),
         _ptr(perm_out), _ptr(count_out), _ptr(s), s.numel())


def gather(ctx: Context, perm: torch.Tensor, pairs, n: Optional[int] = None):
    n = int(perm.numel()) if n is None else n
    f = _fields(pairs)
    call("plx_gather", ctx.handle, n, _ptr(perm), f, len(pairs))


def radix_sort_u32(ctx: Context, keys: torch.Tensor, keys_out: torch.Tensor,
                   perm_out: torch.Tensor, begin_bit: int = 0, end_bit: int = 32, *,
                   scratch: Optional[Scratch] = None):
    n = int(keys.numel())
    nbytes = _abi.lib().plx_radix_sort_scratch_bytes(n)
    s = (scratch or Scratch(ctx.device)).get(nbytes)
    call("plx_radix_sort_u32", ctx.handle, n, _ptr(keys), _ptr(keys_out), _ptr(perm_out),
         begin_bit, end_bit, _ptr(s), s.numel())


def sort_tail_u32(ctx: Context, keys: torch.Tensor, n_sorted: torch.Tensor,
                  keys_out: torch.Tensor, perm_out: torch.Tensor, begin_bit: int = 0,
                  end_bit: int = 32, *, scratch: Optional[Scratch] = None):
    """``radix_sort_u32`` for keys whose first ``n_sorted`` (a one-element
    int64 DEVICE tensor, e.g. a compaction's count) are already in order:
    the tail is sorted and merged in; the same output bit for bit."""
    n = int(keys.numel())
    nbytes = _abi.lib().plx_sort_tail_scratch_bytes(n)
    s = (scratch or Scratch(ctx.device)).get(nbytes)
    call("plx_sort_tail_u32", ctx.handle, n, _ptr(n_sorted), _ptr(keys), _ptr(keys_out),
         _ptr(perm_out), begin_bit, end_bit, _ptr(s), s.numel())


def recompute_levels(ctx: Context, n_units: int, n_input: int, from_id: torch.Tensor,
                     to_id: torch.Tensor, level: torch.Tensor, *,
                     dead: Optional[torch.Tensor] = None, rounds: Optional[torch.Tensor] = None,
                     scratch: Optional[Scratch] = None) -> None:
    """RecomputeLevels (plastix.hpp:466-537) on the device: ``level`` (int16
    tensor holding the uint16 levels of all ``n_units`` units) is reset for
    the non-input units and refilled by the level-parallel Kahn pass over the
    live connections. ``rounds`` (optional 1-element int32 device tensor)
    receives the number of non-empty frontiers."""
    n = int(from_id.numel())
    nbytes = _abi.lib().plx_recompute_levels_scratch_bytes(n_units, n)
    s = (scratch or Scratch(ctx.device)).get(nbytes)
    call("plx_recompute_levels", ctx.handle, n_units, n_input, n, _ptr(from_id) if n else None,
         _ptr(to_id) if n else None, _ptr(dead) if n else None, _ptr(level) if n_units else None,
         _ptr(rounds), _ptr(s), s.numel())


def sort_connections_by_level(ctx: Context, n_units: int, n_input: int,
                              from_id: torch.Tensor, to_id: torch.Tensor, level: torch.Tensor,
                              pairs, *, dead: Optional[torch.Tensor] = None,
                              scratch: Optional[Scratch] = None):
    """SortConnectionsByLevel (plastix.hpp:539-579) on the device: recompute
    the unit levels, refresh SrcLevel = level[FromId], stable radix sort of the
    connections on the 16-bit SrcLevel, Gather of every field in ``pairs``
    ((src, dst) tensors; include FromId, ToId and Dead there to move them).
    Returns (perm, sorted SrcLevel as int16, NumLevels as a 1-element int32
    device tensor: the largest SrcLevel + 1, 0 without connections)."""
    n = int(from_id.numel())
    dev = from_id.device
    recompute_levels(ctx, n_units, n_input, from_id, to_id, level, dead=dead, scratch=scratch)
    src_level = torch.empty(n, dtype=torch.int16, device=dev)
    if n:
        call("plx_src_levels", ctx.handle, n, _ptr(from_id), _ptr(level), n_units,
             _ptr(src_level))
    keys = src_level.to(torch.int32)
    keys_out = torch.empty(n, dtype=torch.int32, device=dev)
    perm = torch.empty(n, dtype=torch.int32, device=dev)
    num_levels = torch.zeros(1, dtype=torch.int32, device=dev)
    if n:
        radix_sort_u32(ctx, keys, keys_out, perm, 0, 16, scratch=scratch)
        sorted_level = torch.empty_like(src_level)
        gather(ctx, perm, list(pairs) + [(src_level, sorted_level)])
        num_levels.copy_((keys_out[n - 1:] & 0xFFFF) + 1)
    else:
        sorted_level = src_level
    return perm, sorted_level, num_levels


def sort_unique_u64(ctx: Context, keys: torch.Tensor, out: torch.Tensor,
                    count_out: torch.Tensor, *, scratch: Optional[Scratch] = None) -> None:
    """Proposal commit: distinct keys of ``keys`` (int64 tensor holding the
    uint64 (To << 32 | From) bits) in ascending unsigned order into ``out``;
    their number into ``count_out`` (1-element int64 device tensor)."""
    n = int(keys.numel())
    nbytes = _abi.lib().plx_sort_unique_u64_scratch_bytes(n)
    s = (scratch or Scratch(ctx.device)).get(nbytes)
    call("plx_sort_unique_u64", ctx.handle, n, _ptr(keys) if n else None,
         _ptr(out) if n else None, _ptr(count_out), _ptr(s), s.numel())


def regrow(ctx: Context, count: torch.Tensor, from_id: torch.Tensor, to_id: torch.Tensor,
           weight: Optional[torch.Tensor], age: Optional[torch.Tensor], *, src_base: int,
           n_src: int, dst_base: int, n_dst: int, seed: int, step_base: int):
    call("plx_regrow", ctx.handle, int(from_id.numel()), _ptr(count), _ptr(from_id),
         _ptr(to_id), _ptr(weight), _ptr(age), src_base, n_src, dst_base, n_dst, seed,
         step_base)


class StructuralLayer:
    """Sparse layer with structural plasticity, stepped entirely on the device:
    prune connections with |w| < threshold (order-preserving compaction, ages
    of survivors +1), regrow the same number with seeded random endpoints
    (w = 0, age = 0), re-sort all connections by ToId (the regrown tail
    radix-sorted and merged with the still-sorted survivors: a stable sort +
    Gather), rebuild the row offsets and run the forward sweep (one thread per
    row: two connections per destination at the benchmark's shape). Sources
    are units [0, n_src), destinations [n_src, n_src + n_dst)."""

    def __init__(self, ctx: Context, n_src: int, n_dst: int, from_id, to_id, weight, age,
                 *, threshold: float = 0.02, seed: int = 1):
        dev = ctx.device
        self.ctx, self.n_src, self.n_dst = ctx, n_src, n_dst
        self.threshold, self.seed = threshold, seed
        n = int(from_id.numel())
        self.n = n
        mk = lambda t, dt: t.to(dev, dt).contiguous().clone()  # noqa: E731
        self.f, self.t = mk(from_id, torch.int32), mk(to_id, torch.int32)
        self.w, self.age = mk(weight, torch.float32), mk(age, torch.uint8)
        self.f2, self.t2 = torch.empty_like(self.f), torch.empty_like(self.t)
        self.w2, self.age2 = torch.empty_like(self.w), torch.empty_like(self.age)
        self.keys_sorted = torch.empty_like(self.t)
        self.perm = torch.empty_like(self.t)
        self.count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.scratch = Scratch(dev)
        self.act_dst = torch.zeros(n_dst, dtype=torch.float32, device=dev)
        # ToId itself is the sort key (the same stable order as ToId - n_src),
        # on the bits its largest value needs
        self.key_bits = max(1, (n_src + n_dst - 1).bit_length())
        self.step_index = 0
        # a structural layer has a few connections per destination: its
        # forward sweep is the row-per-thread fold over row offsets alone
        self.row_ptr = torch.empty(n_dst + 1, dtype=torch.int32, device=dev)
        self._index()

    def _index(self):
        call("plx_csr_row_ptr", self.ctx.handle, _ptr(self.t), self.n, self.n_src, self.n_dst,
             _ptr(self.row_ptr))

    def _state_tensors(self):
        return {"from_id": self.f, "to_id": self.t, "weight": self.w, "age": self.age,
                "act_dst": self.act_dst}

    def _state_meta(self):
        return {"step_index": self.step_index}

    def _load_meta(self, meta):
        self.step_index = int(meta["step_index"])
        self._index()

    def save(self, path) -> None:
        """Checkpoint: the connection fields, destination activations and the
        step counter that seeds regrowth."""
        from .checkpoint import save_state
        save_state(self, path)

    def load(self, path) -> None:
        from .checkpoint import load_state
        load_state(self, path)

    def step(self, act_src: torch.Tensor) -> torch.Tensor:
        ctx = self.ctx
        compact(ctx, self.n, _abi.KEEP_ABS_GE, self.w,
                [(self.f, self.f2), (self.t, self.t2), (self.w, self.w2),
                 (self.age, self.age2)], self.count, threshold=self.threshold,
                flags=[0, 0, 0, _abi.FIELD_INC_SAT_U8], scratch=self.scratch)
        regrow(ctx, self.count, self.f2, self.t2, self.w2, self.age2, src_base=0,
               n_src=self.n_src, dst_base=self.n_src, n_dst=self.n_dst, seed=self.seed,
               step_base=self.step_index * self.n)
        # survivors are still in destination order: sort the regrown tail
        # and merge it in (the same permutation as a full stable sort)
        sort_tail_u32(ctx, self.t2, self.count, self.keys_sorted, self.perm, 0, self.key_bits,
                      scratch=self.scratch)
        # the sorted keys are the re-sorted ToId field itself: only the other
        # fields are gathered
        self.t, self.keys_sorted = self.keys_sorted, self.t
        gather(ctx, self.perm, [(self.f2, self.f), (self.w2, self.w), (self.age2, self.age)])
        self._index()
        sweep_forward_rows(ctx, self.row_ptr, self.f, self.w, act_src, self.act_dst)
        self.step_index += 1
        return self.act_dst


# ---------------------------------------------------------------------------
# SwiftTD (examples/swifttd/swifttd.cpp): N features -> one value unit
# ---------------------------------------------------------------------------
TD_FIELDS = ("w", "z", "z_delta", "delta_w", "h", "h_old", "h_temp", "z_bar", "p", "beta")
TD_GLOBALS = ("gamma", "lambda", "eta", "eta_min", "decay", "meta",
              "v", "v_old", "delta", "v_delta_prev", "v_delta", "tau", "b")


class SwiftTDLearner:
    """The SwiftTD network of the reference example on the device.

    State is the reference's ten connection fields (swifttd.cpp:199-209) as
    rows of one [10, n] float32 tensor (row stride padded to 16 bytes), plus
    the 13-float globals record (swifttd.cpp:47-62) in device memory.
    ``step(active_idx, reward)`` is one Network::DoStep with the given active
    features (sorted, unique, int32 device tensor) and a device reward scalar;
    it returns V (a 1-element device tensor). ``alpha_init`` sets Beta =
    log(alpha_init) as SwiftTDConnInit does (swifttd.cpp:66-72).
    """

    def __init__(self, ctx: Context, n_features: int, *, gamma=0.99, lambda_=0.9, eta=0.05,
                 eta_min=1e-7, decay=0.999, meta=1e-3, alpha_init=0.05,
                 max_active: Optional[int] = None):
        import math
        import struct

        self.ctx = ctx
        self.n = int(n_features)
        dev = ctx.device
        self.stride = (self.n + 3) // 4 * 4
        self.state = torch.zeros((len(TD_FIELDS), self.stride), dtype=torch.float32, device=dev)
        # std::log on a float argument, rounded to float (SwiftTDConnInit).
        a32 = struct.unpack("f", struct.pack("f", alpha_init))[0]
        self.state[9].fill_(struct.unpack("f", struct.pack("f", math.log(a32)))[0])
        self.globals = torch.zeros(len(TD_GLOBALS), dtype=torch.float32, device=dev)
        self.globals[:6] = torch.tensor([gamma, lambda_, eta, eta_min, decay, meta],
                                        dtype=torch.float32)
        self.v = torch.zeros(1, dtype=torch.float32, device=dev)
        self.max_active = int(max_active if max_active is not None else max(1, self.n // 100))
        nbytes = _abi.lib().plx_swifttd_scratch_bytes(self.n, self.max_active)
        self.scratch = torch.zeros(int(nbytes), dtype=torch.uint8, device=dev)
        self._ptrs = (c_void_p * len(TD_FIELDS))(
            *[self.state[i].data_ptr() for i in range(len(TD_FIELDS))])

    def field(self, name: str) -> torch.Tensor:
        return self.state[TD_FIELDS.index(name), :self.n]

    def _state_tensors(self):
        return {"state": self.state, "globals": self.globals, "v": self.v}

    def save(self, path) -> None:
        """Checkpoint: the ten connection fields, the globals record, V."""
        from .checkpoint import save_state
        save_state(self, path)

    def load(self, path) -> None:
        from .checkpoint import load_state
        load_state(self, path)

    def fields(self) -> torch.Tensor:
        return self.state[:, :self.n]

    def step(self, active_idx: torch.Tensor, reward: torch.Tensor,
             active_val: Optional[torch.Tensor] = None) -> torch.Tensor:
        k = int(active_idx.numel())
        if k > self.max_active:
            nbytes = _abi.lib().plx_swifttd_scratch_bytes(self.n, k)
            self.scratch = torch.zeros(int(nbytes), dtype=torch.uint8,
                                       device=self.scratch.device)
            self.max_active = k
        call("plx_swifttd_step", self.ctx.handle, self.n, self._ptrs,
             _ptr(active_idx) if k else None, _ptr(active_val), k, _ptr(reward),
             _ptr(self.globals), _ptr(self.v), _ptr(self.scratch), self.scratch.numel())
        return self.v

    def step_parts(self, active_idx: torch.Tensor, reward: torch.Tensor,
                   active_val: Optional[torch.Tensor] = None, between=None) -> torch.Tensor:
        """``step`` as its two halves (active-set reductions, then the dense
        pass), calling ``between()`` in between (e.g. to record an event)."""
        k = int(active_idx.numel())
        if k > self.max_active:
            raise ValueError("more active features than max_active")
        idx = _ptr(active_idx) if k else None
        call("plx_swifttd_reduce", self.ctx.handle, self.n, self._ptrs, idx, _ptr(active_val),
             k, _ptr(reward), _ptr(self.globals), _ptr(self.v), _ptr(self.scratch),
             self.scratch.numel())
        if between is not None:
            between()
        call("plx_swifttd_apply", self.ctx.handle, self.n, self._ptrs, idx, _ptr(active_val), k,
             _ptr(self.globals), _ptr(self.scratch), self.scratch.numel())
        return self.v


# ---------------------------------------------------------------------------
# Backward sweep (K2): a source-major copy of a connection range
# ---------------------------------------------------------------------------
class SrcMajor:
    """Source-major order of connections whose sources are units
    [src_base, src_base + n_src): the permutation from plx_transpose, a CSR
    over the sources, and the gathered ToId (the index the backward sweep
    gathers through) and Weight. ``reverse`` gives each source's
    connections in descending index order (Pipeline backward,
    plastix.hpp:193-203); otherwise ascending (Topological,
    plastix.hpp:172-181). Connections from other units are left out."""

    def __init__(self, ctx: Context, from_id: torch.Tensor, to_id: torch.Tensor,
                 weight: torch.Tensor, src_base: int, n_src: int, reverse: bool):
        n = int(from_id.numel())
        dev = ctx.device
        self.ctx = ctx
        keys = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        self.perm = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        row_ptr = torch.empty(n_src + 1, dtype=torch.int32, device=dev)
        nbytes = _abi.lib().plx_transpose_scratch_bytes(n)
        scratch = torch.empty(int(nbytes), dtype=torch.uint8, device=dev)
        call("plx_transpose", ctx.handle, n, _ptr(from_id) if n else None, src_base, n_src,
             int(reverse), _ptr(keys), _ptr(self.perm), _ptr(row_ptr), _ptr(scratch),
             scratch.numel())
        del scratch, keys
        self.csr = DstCsr.from_row_ptr(ctx, row_ptr)
        self.m = self.csr.n_edges
        self.src_base, self.n_src = src_base, n_src
        self.to_id = torch.empty(max(self.m, 1), dtype=torch.int32, device=dev)
        self.weight = torch.empty(max(self.m, 1), dtype=torch.float32, device=dev)
        if self.m:
            gather(ctx, self.perm, [(to_id, self.to_id), (weight, self.weight)], n=self.m)

    def refresh_weight(self, weight: torch.Tensor) -> None:
        """Re-gathers Weight (after an update of the destination-major copy)."""
        if self.m:
            gather(self.ctx, self.perm, [(weight, self.weight)], n=self.m)

    def backward(self, dval: torch.Tensor, out_rows: torch.Tensor, value_rows: torch.Tensor,
                 apply: int) -> None:
        """out_rows[s] = Apply(fold over source s of Weight * dval[ToId])."""
        sweep_forward(self.ctx, self.csr, self.to_id, self.weight, dval, out_rows,
                      apply=apply, value=value_rows)


class MlpTopoNet:
    """The mlp_xor.cpp network on the device: FullyConnected sigmoid layers
    in the reference's Topological mode (levels processed in order), MSELoss,
    the sigmoid backward pass and the gradient-descent connection update --
    one Network::DoStep per ``step``. Connections are stored per level
    (SrcLevel), destination-major as FullyConnected creates them."""

    def __init__(self, ctx: Context, layers, weights, lr: float = 0.5):
        import numpy as np

        self.ctx = ctx
        self.layers = [int(x) for x in layers]
        self.begin = [0]
        for n in self.layers:
            self.begin.append(self.begin[-1] + n)
        self.n_units = self.begin[-1]
        self.lr = float(lr)
        dev = ctx.device
        w_all = np.asarray(weights, np.float32)
        self.from_id, self.to_id, self.w, self.csr, self.bwd = [], [], [], [], {}
        off = 0
        for L in range(1, len(self.layers)):
            frm = np.repeat(np.arange(self.begin[L - 1], self.begin[L], dtype=np.int32)[None, :],
                            self.layers[L], axis=0).reshape(-1)
            to = np.repeat(np.arange(self.begin[L], self.begin[L + 1], dtype=np.int32),
                           self.layers[L - 1])
            m = frm.size
            f_d = torch.from_numpy(frm).to(dev)
            t_d = torch.from_numpy(to).to(dev)
            w_d = torch.from_numpy(w_all[off:off + m].copy()).to(dev)
            off += m
            self.from_id.append(f_d)
            self.to_id.append(t_d)
            self.w.append(w_d)
            self.csr.append(DstCsr(ctx, t_d, self.begin[L], self.layers[L], use_to_id=False))
        for L in range(1, len(self.layers) - 1):  # backward levels (SrcLevel == L)
            self.bwd[L] = SrcMajor(ctx, self.from_id[L], self.to_id[L], self.w[L],
                                   self.begin[L], self.layers[L], reverse=False)
        self.act = torch.zeros(self.n_units, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(self.n_units, dtype=torch.float32, device=dev)

    def weights(self) -> torch.Tensor:
        return torch.cat(self.w)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """DoForwardPass (Topological: level by level, sigmoid Apply)."""
        self.act[:self.layers[0]].copy_(x)
        for L in range(1, len(self.layers)):
            b0, b1 = self.begin[L], self.begin[L + 1]
            sweep_forward(self.ctx, self.csr[L - 1], self.from_id[L - 1], self.w[L - 1],
                          self.act, self.act[b0:b1], apply=_abi.APPLY_SIGMOID)
        return self.act[self.begin[-2]:]

    def step(self, x: torch.Tensor, target: torch.Tensor) -> None:
        self.forward(x)
        top = len(self.layers) - 1
        o0, o1 = self.begin[top], self.begin[top + 1]
        call("plx_mse_sigmoid_grad", self.ctx.handle, o1 - o0, _ptr(self.act[o0:o1]),
             _ptr(target), _ptr(self.grad[o0:o1]))
        for L in range(top - 1, 0, -1):
            b0, b1 = self.begin[L], self.begin[L + 1]
            sm = self.bwd[L]
            sm.refresh_weight(self.w[L])
            sm.backward(self.grad, self.grad[b0:b1], self.act[b0:b1], _abi.APPLY_SIGMOID_GRAD)
        for L in range(1, len(self.layers)):
            b0, b1 = self.begin[L], self.begin[L + 1]
            sweep_update(self.ctx, self.csr[L - 1], self.from_id[L - 1], self.act,
                         self.grad[b0:b1], self.w[L - 1], self.w[L - 1],
                         kind=_abi.UPDATE_GRADIENT, rate=self.lr)


class ChunkedRows:
    """Connections of a row set in the chunked-source layout (see
    plx_chunked_build): rows are units [row_base, row_base + n_rows), the
    gathered side units [src_base, src_base + n_src). ``weight`` is the
    layout-order weight copy (padding 0); ``perm`` maps layout slots to the
    original connection index (-1 for padding)."""

    def __init__(self, ctx: Context, gather_id: torch.Tensor, row_id: torch.Tensor,
                 weight: torch.Tensor, src_base: int, n_src: int, row_base: int, n_rows: int):
        lib = _abi.lib()
        n = int(gather_id.numel())
        dev = ctx.device
        self.ctx = ctx
        self.n_pad_max = int(lib.plx_chunked_max_padded(n, n_rows, n_src))
        n_chunks = (n_src + _abi.CHUNK_SOURCES - 1) // _abi.CHUNK_SOURCES
        self.seg_ptr = torch.empty(n_chunks * n_rows + 1, dtype=torch.int32, device=dev)
        self.src = torch.empty(self.n_pad_max, dtype=torch.int16, device=dev)
        self.perm = torch.empty(self.n_pad_max, dtype=torch.int32, device=dev)
        scratch = torch.empty(int(lib.plx_chunked_scratch_bytes(n, n_rows, n_src)),
                              dtype=torch.uint8, device=dev)
        call("plx_chunked_build", ctx.handle, n, _ptr(gather_id) if n else None, src_base, n_src,
             _ptr(row_id) if n else None, row_base, n_rows, _ptr(self.seg_ptr), _ptr(self.src),
             _ptr(self.perm), _ptr(scratch), scratch.numel())
        del scratch
        self.weight = torch.zeros(self.n_pad_max, dtype=torch.float32, device=dev)
        if n:
            call("plx_chunked_gather", ctx.handle, self.n_pad_max, _ptr(self.perm),
                 _ptr(weight), _ptr(self.weight))
        self.partial = torch.empty(max(n_chunks * n_rows, 1), dtype=torch.float32, device=dev)
        self.struct = Chunked(_ptr(self.seg_ptr), _ptr(self.src), _ptr(self.perm), n_rows, n_src,
                              n_chunks)
        self.src_base, self.n_src, self.row_base, self.n_rows = src_base, n_src, row_base, n_rows

    def fold(self, gathered: torch.Tensor, out: torch.Tensor, apply: int,
             value: Optional[torch.Tensor] = None) -> None:
        """out[r] = Apply(sum of weight * gathered[src] over row r, value[r]);
        gathered holds the n_src values of the gathered range."""
        call("plx_chunked_fold", self.ctx.handle, byref(self.struct), _ptr(self.weight),
             _ptr(gathered), apply, _ptr(value), _ptr(out), _ptr(self.partial))

    def fold_ipc_value(self, gathered: torch.Tensor, x: torch.Tensor, eps: torch.Tensor,
                       act: torch.Tensor, gamma: float) -> None:
        """An iPC backward block (TANH_GRAD with value x) with the value-node
        update of its rows fused in: x += gamma * (-eps + bu); act = tanh(x)."""
        call("plx_chunked_fold_ipc_value", self.ctx.handle, byref(self.struct),
             _ptr(self.weight), _ptr(gathered), _ptr(x), _ptr(eps), gamma, _ptr(act),
             _ptr(self.partial))

    def update(self, gathered: torch.Tensor, row_val: torch.Tensor, kind: int,
               rate: float) -> None:
        call("plx_chunked_update", self.ctx.handle, byref(self.struct), _ptr(self.weight),
             _ptr(gathered), _ptr(row_val), kind, rate)

    def weights_in_original_order(self, n: int) -> torch.Tensor:
        """The layout's weights scattered back to connection order (tests)."""
        out = torch.zeros(n, dtype=torch.float32, device=self.weight.device)
        valid = self.perm >= 0
        out[self.perm[valid].long()] = self.weight[valid]
        return out


class PredictiveCodingNet:
    """Streaming iPC (examples/ipc-multilayer/ipc_multilayer.cpp) on a stack
    of sparse layers: layer 0 takes the input, the last layer is the output,
    the ones between are tanh hidden layers with persistent value nodes.
    Block l holds the connections into layer l + 1 (destination-major, the
    reference's connection order); blocks whose sources are hidden also keep
    a source-major copy (descending per source: the Pipeline backward order)
    with its own weights, updated with the same rule and rounding so both
    copies stay identical.

    ``iteration()`` is one inference step of iPCStep (pre-step done by the
    previous value update, DoForwardPass with eps = x - mu, DoBackwardPass
    with the bottom-up Apply, value-node update). ``update()`` is
    DoUpdateConnectionState (theta += alpha * eps * f(x_src)).
    ``example_step()`` is the example's own order: forward, backward, update,
    value update."""

    def __init__(self, ctx: Context, sizes, blocks, *, gamma: float = 0.1,
                 alpha: float = 0.005, layout: str = "csr"):
        """blocks[l] = (from_id, to_id, weight) device tensors of the
        connections into layer l + 1 (absolute unit ids, destination-major).
        layout "csr": destination-major CSR sweeps and source-major copies
        (exact left folds for rows up to PLX_SEQ_ROW_MAX); layout "chunked":
        the chunked-source layout for both directions (for long rows such as
        2,048 fan-in; folds in a fixed chunked order)."""
        self.ctx = ctx
        self.sizes = [int(s) for s in sizes]
        self.begin = [0]
        for s in self.sizes:
            self.begin.append(self.begin[-1] + s)
        self.n_units = self.begin[-1]
        self.gamma, self.alpha = float(gamma), float(alpha)
        dev = ctx.device
        self.layout = layout
        self.from_id, self.w, self.csr, self.sm = [], [], [], {}
        self.fwd, self.bwd = [], {}
        for l, (f, t, w) in enumerate(blocks):
            if layout == "chunked":
                self.fwd.append(ChunkedRows(ctx, f, t, w, self.begin[l], self.sizes[l],
                                            self.begin[l + 1], self.sizes[l + 1]))
                if l >= 1:
                    self.bwd[l] = ChunkedRows(ctx, t, f, w, self.begin[l + 1], self.sizes[l + 1],
                                              self.begin[l], self.sizes[l])
                continue
            self.from_id.append(f)
            self.w.append(w)
            self.csr.append(DstCsr(ctx, t, self.begin[l + 1], self.sizes[l + 1],
                                   use_to_id=False))
            if l >= 1:
                self.sm[l] = SrcMajor(ctx, f, t, w, self.begin[l], self.sizes[l], reverse=True)
        self.x = torch.zeros(self.n_units, dtype=torch.float32, device=dev)
        self.act = torch.zeros_like(self.x)
        self.err = torch.zeros_like(self.x)
        self.bu = torch.zeros_like(self.x)

    @property
    def hidden(self):
        return self.begin[1], self.begin[-2]

    def _state_tensors(self):
        t = {"x": self.x, "act": self.act, "err": self.err, "bu": self.bu}
        if self.layout == "chunked":
            for l, rows in enumerate(self.fwd):
                t[f"w_fwd{l}"] = rows.weight
            for l, rows in self.bwd.items():
                t[f"w_bwd{l}"] = rows.weight
        else:
            for l, w in enumerate(self.w):
                t[f"w{l}"] = w
            for l, sm in self.sm.items():
                t[f"w_src_major{l}"] = sm.weight
        return t

    def save(self, path) -> None:
        """Checkpoint: value nodes, activations, errors, bottom-up sums and
        every weight copy (both orders) in this network's layout."""
        from .checkpoint import save_state
        save_state(self, path)

    def load(self, path) -> None:
        from .checkpoint import load_state
        load_state(self, path)

    def clamp(self, inputs: torch.Tensor, targets: torch.Tensor) -> None:
        """Clamps the input and output value nodes (ipc_multilayer.cpp:299-304)
        and runs the pre-step (Activation = f(x): inputs identity, hidden
        tanh)."""
        n_in = self.sizes[0]
        self.x[:n_in].copy_(inputs)
        self.act[:n_in].copy_(inputs)
        self.x[self.begin[-2]:].copy_(targets)
        lo, hi = self.hidden
        call("plx_ipc_value_update", self.ctx.handle, hi - lo, _ptr(self.x[lo:hi]), None, None,
             0.0, _ptr(self.act[lo:hi]), 0)

    def _layer(self, t: torch.Tensor, l: int) -> torch.Tensor:
        return t[self.begin[l]:self.begin[l + 1]]

    def forward(self) -> None:
        if self.layout == "chunked":
            for l, ch in enumerate(self.fwd):
                ch.fold(self._layer(self.act, l), self._layer(self.err, l + 1),
                        _abi.APPLY_IPC_ERROR, value=self._layer(self.x, l + 1))
            return
        for l in range(len(self.csr)):
            b0, b1 = self.begin[l + 1], self.begin[l + 2]
            sweep_forward(self.ctx, self.csr[l], self.from_id[l], self.w[l], self.act,
                          apply=_abi.APPLY_IPC_ERROR, value=self.x[b0:b1],
                          err_out=self.err[b0:b1])

    def backward(self) -> None:
        if self.layout == "chunked":
            for l, ch in self.bwd.items():
                ch.fold(self._layer(self.err, l + 1), self._layer(self.bu, l),
                        _abi.APPLY_TANH_GRAD, value=self._layer(self.x, l))
            return
        for l, sm in self.sm.items():
            b0, b1 = self.begin[l], self.begin[l + 1]
            sm.backward(self.err, self.bu[b0:b1], self.x[b0:b1], _abi.APPLY_TANH_GRAD)

    def value_update(self) -> None:
        lo, hi = self.hidden
        call("plx_ipc_value_update", self.ctx.handle, hi - lo, _ptr(self.x[lo:hi]),
             _ptr(self.err[lo:hi]), _ptr(self.bu[lo:hi]), self.gamma, _ptr(self.act[lo:hi]), 1)

    def update(self) -> None:
        if self.layout == "chunked":
            for l, ch in enumerate(self.fwd):
                ch.update(self._layer(self.act, l), self._layer(self.err, l + 1),
                          _abi.UPDATE_HEBBIAN, self.alpha)
                if l in self.bwd:
                    self.bwd[l].update(self._layer(self.err, l + 1), self._layer(self.act, l),
                                       _abi.UPDATE_HEBBIAN_T, self.alpha)
            return
        for l in range(len(self.csr)):
            b0, b1 = self.begin[l + 1], self.begin[l + 2]
            sweep_update(self.ctx, self.csr[l], self.from_id[l], self.act, self.err[b0:b1],
                         self.w[l], self.w[l], kind=_abi.UPDATE_HEBBIAN, rate=self.alpha)
            if l in self.sm:
                sm = self.sm[l]
                s0, s1 = self.begin[l], self.begin[l + 1]
                sweep_update(self.ctx, sm.csr, sm.to_id, self.err, self.act[s0:s1],
                             sm.weight, sm.weight, kind=_abi.UPDATE_HEBBIAN_T,
                             rate=self.alpha)

    def weights(self, l: int, n: Optional[int] = None) -> torch.Tensor:
        """Block l's weights in connection order."""
        if self.layout == "chunked":
            return self.fwd[l].weights_in_original_order(n)
        return self.w[l]

    def iteration(self) -> None:
        self.forward()
        if self.layout == "chunked":
            # the value-node update runs in the backward folds' epilogue:
            # nothing reads x or act between the two in an inference step
            for l, ch in self.bwd.items():
                ch.fold_ipc_value(self._layer(self.err, l + 1), self._layer(self.x, l),
                                  self._layer(self.err, l), self._layer(self.act, l),
                                  self.gamma)
            return
        self.backward()
        self.value_update()

    def example_step(self) -> None:
        self.forward()
        self.backward()
        self.update()
        self.value_update()
