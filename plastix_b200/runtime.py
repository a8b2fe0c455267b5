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
from ._abi import Csr, call


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

    def __init__(self, ctx: Context, to_id: torch.Tensor, row_base: int, n_rows: int):
        n_edges = int(to_id.numel())
        self.row_ptr = torch.empty(n_rows + 1, dtype=torch.int32, device=ctx.device)
        call("plx_csr_row_ptr", ctx.handle, c_void_p(_ptr(to_id) if n_edges else None),
             n_edges, row_base, n_rows, c_void_p(_ptr(self.row_ptr)))
        self._init_plan(ctx, n_edges, n_rows)

    @classmethod
    def from_row_ptr(cls, ctx: Context, row_ptr: torch.Tensor) -> "DstCsr":
        self = cls.__new__(cls)
        self.row_ptr = row_ptr.to(device=ctx.device, dtype=torch.int32).contiguous()
        n_rows = int(self.row_ptr.numel()) - 1
        n_edges = int(self.row_ptr[-1].item())
        self._init_plan(ctx, n_edges, n_rows)
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


class HebbianSweepLayer:
    """One sparse layer stepped like ``Network::DoStep`` in Pipeline mode with
    the Hebbian trace rule: forward sum (identity Apply) + per-connection
    trace/weight update, fused into one pass. Weights and traces are
    double-buffered on the device (the fused sweep reads one copy and writes
    the other); ``weight``/``trace`` are the current copies."""

    def __init__(self, ctx: Context, n_src: int, n_dst: int, from_id: torch.Tensor,
                 to_id: torch.Tensor, weight: torch.Tensor,
                 trace: Optional[torch.Tensor] = None, *, decay: float = 0.9,
                 rate: float = 1e-3, dead: Optional[torch.Tensor] = None):
        dev = ctx.device
        self.ctx = ctx
        self.n_src, self.n_dst = n_src, n_dst
        self.decay, self.rate = decay, rate
        self.from_id = from_id.to(dev, torch.int32).contiguous()
        self.to_id = to_id.to(dev, torch.int32).contiguous()
        self.dead = None if dead is None else dead.to(dev, torch.uint8).contiguous()
        n = self.from_id.numel()
        self._w = [weight.to(dev, torch.float32).contiguous().clone(),
                   torch.empty(n, dtype=torch.float32, device=dev)]
        tr = torch.zeros(n, dtype=torch.float32, device=dev) if trace is None else \
            trace.to(dev, torch.float32).contiguous().clone()
        self._e = [tr, torch.empty(n, dtype=torch.float32, device=dev)]
        self._cur = 0
        self.csr = DstCsr(ctx, self.to_id, n_src, n_dst)
        self.act_dst = torch.zeros(n_dst, dtype=torch.float32, device=dev)

    @property
    def weight(self) -> torch.Tensor:
        return self._w[self._cur]

    @property
    def trace(self) -> torch.Tensor:
        return self._e[self._cur]

    def step(self, act_src: torch.Tensor) -> torch.Tensor:
        c, o = self._cur, 1 - self._cur
        sweep_forward_hebbian(self.ctx, self.csr, self.from_id, act_src, self._w[c],
                              self._w[o], self._e[c], self._e[o], self.act_dst,
                              decay=self.decay, rate=self.rate, dead=self.dead)
        self._cur = o
        return self.act_dst
