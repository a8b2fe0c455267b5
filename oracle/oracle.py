"""numpy front end of the oracle (test infrastructure only).

Loads ``oracle/libplx_oracle.so`` (the C restatement) and, when present,
``oracle/_ref/libplx_ref.so`` (the reference compiled from its own sources).
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module; it is the checker, never the thing measured or shipped.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libplx_oracle.so"
REF_SO = HERE / "_ref" / "libplx_ref.so"

_orc = None
_ref = None


def _p(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(c_void_p)


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            from oracle import build as _b
            _b.build_oracle()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.oracle_forward_pipeline.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_void_p, c_uint64, c_uint64,
                                              c_int, c_void_p, c_void_p, c_void_p]
        L.oracle_update_hebbian_trace.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p,
                                                  c_void_p, c_void_p, c_void_p, c_float,
                                                  c_float]
        L.oracle_update_post.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_int, c_float, c_void_p]
        L.oracle_step_hebbian.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_uint64, c_uint64, c_float,
                                          c_float, c_void_p]
        L.oracle_gather.argtypes = [c_void_p, c_uint64, c_void_p, c_void_p, c_uint32]
        L.oracle_survivors.argtypes = [c_void_p, c_uint64, c_void_p]
        L.oracle_survivors.restype = c_uint64
        L.oracle_stable_sort_u32.argtypes = [c_void_p, c_uint64, c_void_p]
        L.oracle_sort_unique_u64.argtypes = [c_void_p, c_uint64, c_void_p]
        L.oracle_sort_unique_u64.restype = c_uint64
        L.oracle_mix64.argtypes = [c_uint64]
        L.oracle_mix64.restype = c_uint64
        L.oracle_regrow.argtypes = [c_uint64, c_uint64, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_uint32, c_uint32, c_uint32, c_uint32,
                                    c_uint64, c_uint64]
        L.oracle_keep_abs_ge.argtypes = [c_void_p, c_uint64, c_float, c_void_p]
        L.oracle_backward.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_int, c_uint64, c_uint64, c_uint64, c_int,
                                      c_void_p, c_void_p, c_void_p]
        L.oracle_ipc_value_update.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p, c_float,
                                              c_void_p, c_int]
        L.oracle_mse_sigmoid_grad.argtypes = [c_uint64, c_void_p, c_void_p, c_void_p]
        L.oracle_swifttd_step.argtypes = [c_uint64, c_void_p, c_void_p, c_float, c_void_p,
                                          c_int]
        L.oracle_swifttd_step.restype = c_float
        L.oracle_recompute_levels.argtypes = [c_uint32, c_uint32, c_uint64, c_void_p, c_void_p,
                                              c_void_p, c_void_p]
        L.oracle_recompute_levels.restype = ctypes.c_int64
        _orc = L
    return _orc


def ref() -> Optional[ctypes.CDLL]:
    """The reference build, or None when it was not built here."""
    global _ref
    if _ref is None and REF_SO.exists():
        L = ctypes.CDLL(str(REF_SO))
        L.ref_version.restype = ctypes.c_char_p
        L.ref_sweep_run.argtypes = [c_uint64, c_uint64, c_uint64, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_int, c_float, c_float,
                                    c_void_p, c_void_p, c_void_p]
        L.ref_sweep_shards_create.argtypes = [c_uint64, c_uint64, c_uint64, c_void_p,
                                              c_void_p, c_void_p, c_int, c_float, c_float]
        L.ref_sweep_shards_create.restype = c_void_p
        L.ref_sweep_shards_step.argtypes = [c_void_p, c_void_p]
        L.ref_sweep_shards_destroy.argtypes = [c_void_p]
        L.ref_mlp_run.argtypes = [c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_uint64]
        L.ref_mlp_run.restype = ctypes.c_int64
        L.ref_ipc_run.argtypes = [c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_uint64]
        L.ref_ipc_run.restype = ctypes.c_int64
        L.ref_swifttd_example_run.argtypes = [c_uint64, c_void_p, c_void_p, c_int, c_float,
                                              c_void_p, c_void_p]
        if hasattr(L, "ref_structural_run"):
            L.ref_structural_run.argtypes = ([ctypes.c_int] + [c_uint32] * 4 + [ctypes.c_int]
                                             + [c_void_p, c_uint64] + [c_void_p] * 10)
            L.ref_structural_run.restype = c_int
        if hasattr(L, "ref_levels_run"):
            L.ref_levels_run.argtypes = [c_uint64, c_uint64, c_uint64] + [c_void_p] * 8
            L.ref_levels_run.restype = c_int
        _ref = L
    return _ref


# ---------------------------------------------------------------------------
# Forward / update (unit arrays are absolute: inputs then destinations)
# ---------------------------------------------------------------------------
def forward_pipeline(from_id, to_id, w, act, num_input, apply=0, dead=None, value=None):
    """Returns (act, err) after one Pipeline DoForwardPass. act is copied."""
    act = np.array(act, dtype=np.float32, copy=True)
    n_units = act.size
    acc = np.zeros(n_units, np.float32)
    err = np.zeros(n_units, np.float32) if apply == 3 else None
    value = None if value is None else np.ascontiguousarray(value, np.float32)
    orc().oracle_forward_pipeline(from_id.size, _p(from_id), _p(to_id), _p(dead), _p(w),
                                  _p(act), n_units, num_input, apply, _p(value), _p(err),
                                  _p(acc))
    return act, err


def step_hebbian(from_id, to_id, w, trace, act, num_input, decay, rate, sweeps=1,
                 dead=None):
    """`sweeps` Pipeline DoSteps of the Hebbian trace workload. Returns new
    (w, trace, act) arrays; act keeps the inputs in [0, num_input)."""
    w = np.array(w, np.float32, copy=True)
    trace = np.array(trace, np.float32, copy=True)
    act = np.array(act, np.float32, copy=True)
    acc = np.zeros(act.size, np.float32)
    for _ in range(sweeps):
        orc().oracle_step_hebbian(from_id.size, _p(from_id), _p(to_id), _p(dead), _p(w),
                                  _p(trace), _p(act), act.size, num_input, decay, rate,
                                  _p(acc))
    return w, trace, act


def update_post(from_id, to_id, act, post, w, kind, rate, dead=None):
    w = np.array(w, np.float32, copy=True)
    orc().oracle_update_post(from_id.size, _p(from_id), _p(to_id), _p(dead), _p(act),
                             _p(np.ascontiguousarray(post, np.float32)), kind, rate, _p(w))
    return w


# ---------------------------------------------------------------------------
# Permutations (SOAAllocator::Gather semantics)
# ---------------------------------------------------------------------------
def survivors(keep: np.ndarray) -> np.ndarray:
    keep = np.ascontiguousarray(keep, np.uint8)
    perm = np.empty(keep.size, np.uint64)
    m = orc().oracle_survivors(_p(keep), keep.size, _p(perm))
    return perm[:m]


def gather(perm: np.ndarray, field: np.ndarray) -> np.ndarray:
    perm = np.ascontiguousarray(perm, np.uint64)
    field = np.ascontiguousarray(field)
    out = np.empty(perm.size, field.dtype)
    orc().oracle_gather(_p(perm), perm.size, _p(field), _p(out), field.itemsize)
    return out


def stable_sort_perm_u32(keys: np.ndarray) -> np.ndarray:
    keys = np.ascontiguousarray(keys, np.uint32)
    perm = np.empty(keys.size, np.uint64)
    if orc().oracle_stable_sort_u32(_p(keys), keys.size, _p(perm)) != 0:
        raise MemoryError("oracle_stable_sort_u32")
    return perm


def sort_unique_u64(bits: np.ndarray) -> np.ndarray:
    bits = np.array(bits, np.uint64, copy=True)
    out = np.empty(bits.size, np.uint64)
    m = orc().oracle_sort_unique_u64(_p(bits), bits.size, _p(out))
    return out[:m]


# ---------------------------------------------------------------------------
# The reference itself
# ---------------------------------------------------------------------------
def ref_sweep_run(n_src, n_dst, from_id, to_id, w, trace, act_in, sweeps, decay, rate):
    L = ref()
    if L is None:
        raise FileNotFoundError(f"{REF_SO} was not built")
    n = from_id.size
    w_out = np.empty(n, np.float32)
    e_out = np.empty(n, np.float32)
    a_out = np.empty(n_dst, np.float32)
    rc = L.ref_sweep_run(n_src, n_dst, n, _p(from_id), _p(to_id), _p(w), _p(trace),
                         _p(act_in), sweeps, decay, rate, _p(w_out), _p(e_out), _p(a_out))
    if rc != 0:
        raise RuntimeError("ref_sweep_run failed")
    return w_out, e_out, a_out


# ---------------------------------------------------------------------------
# Structural plasticity step (prune |w| < thr -> compact, regrow, re-sort by
# ToId, forward sweep), composed from the restated reference primitives.
# ---------------------------------------------------------------------------
def keep_abs_ge(w, thr):
    w = np.ascontiguousarray(w, np.float32)
    keep = np.empty(w.size, np.uint8)
    orc().oracle_keep_abs_ge(_p(w), w.size, thr, _p(keep))
    return keep


def regrow(from_id, to_id, w, age, count, src_base, n_src, dst_base, n_dst, seed,
           step_base):
    """In place on copies; returns (from, to, w, age)."""
    f, t = from_id.copy(), to_id.copy()
    ww, aa = w.copy(), age.copy()
    orc().oracle_regrow(f.size, count, _p(f), _p(t), _p(ww), _p(aa), src_base, n_src,
                        dst_base, n_dst, seed, step_base)
    return f, t, ww, aa


def structural_step(from_id, to_id, w, age, n_src, n_dst, thr, seed, step_base):
    """One step on the oracle side. Inputs are dst-sorted SoA arrays
    (from/to u32 absolute ids, w f32, age u8); sources are units [0, n_src),
    destinations [n_src, n_src + n_dst). Returns the new dst-sorted arrays and
    the survivor count."""
    keep = keep_abs_ge(w, thr)
    perm = survivors(keep)
    m = perm.size
    f = np.concatenate([gather(perm, from_id), np.zeros(from_id.size - m, np.uint32)])
    t = np.concatenate([gather(perm, to_id), np.zeros(to_id.size - m, np.uint32)])
    ww = np.concatenate([gather(perm, w), np.zeros(w.size - m, np.float32)])
    a_s = gather(perm, age).astype(np.uint16)
    aa = np.concatenate([np.minimum(a_s + 1, 255).astype(np.uint8),
                         np.zeros(age.size - m, np.uint8)])
    f, t, ww, aa = regrow(f, t, ww, aa, m, 0, n_src, n_src, n_dst, seed, step_base)
    order = stable_sort_perm_u32(t - np.uint32(n_src))
    return gather(order, f), gather(order, t), gather(order, ww), gather(order, aa), m


# ---------------------------------------------------------------------------
# SwiftTD (examples/swifttd/swifttd.cpp)
# ---------------------------------------------------------------------------
TD_FIELDS = ("w", "z", "z_delta", "delta_w", "h", "h_old", "h_temp", "z_bar", "p", "beta")
TD_GLOBALS = ("gamma", "lambda", "eta", "eta_min", "decay", "meta",
              "v", "v_old", "delta", "v_delta_prev", "v_delta", "tau", "b")


def td_globals(gamma=0.99, lambda_=0.9, eta=0.05, eta_min=1e-7, decay=0.999, meta=1e-3):
    """A 13-float globals record: hyperparameters, then V, VOld, Delta,
    VDeltaPrev, VDelta, Tau, B (all zero)."""
    g = np.zeros(len(TD_GLOBALS), np.float32)
    g[:6] = (gamma, lambda_, eta, eta_min, decay, meta)
    return g


def td_fields(n, alpha_init=0.05):
    """Initial connection fields as SwiftTDConnInit leaves them: all zero but
    Beta = log(alpha_init) (computed in single precision like std::log on a
    float)."""
    f = np.zeros((len(TD_FIELDS), n), np.float32)
    f[9] = np.float32(np.log(np.float64(np.float32(alpha_init))))
    return f


def swifttd_step(fields, features, reward, globals_, acc_f64=False):
    """One DoStep of the SwiftTD network, in place on fields (10 x n float32,
    C order) and globals_ (13 float32). Returns V."""
    assert fields.dtype == np.float32 and fields.flags["C_CONTIGUOUS"]
    assert globals_.dtype == np.float32 and globals_.size == len(TD_GLOBALS)
    n = fields.shape[1]
    rows = (c_void_p * 10)(*[fields[i].ctypes.data for i in range(10)])
    f = np.ascontiguousarray(features, np.float32)
    assert f.size == n
    return orc().oracle_swifttd_step(n, ctypes.cast(rows, c_void_p), _p(f), float(reward),
                                     _p(globals_), int(acc_f64))


def ref_swifttd_example_run(features, rewards, alpha_init=0.05):
    """The reference's own SwiftTD example network (Gamma 1.0 as that file
    fixes it) stepped over features (steps x n) and rewards. Returns
    (fields 10 x n, V per step)."""
    L = ref()
    if L is None:
        raise FileNotFoundError(f"{REF_SO} was not built")
    feats = np.ascontiguousarray(features, np.float32)
    steps, n = feats.shape
    rw = np.ascontiguousarray(rewards, np.float32)
    fields = np.empty((len(TD_FIELDS), n), np.float32)
    v = np.empty(steps, np.float32)
    if L.ref_swifttd_example_run(n, _p(feats), _p(rw), steps, alpha_init, _p(fields),
                                 _p(v)) != 0:
        raise RuntimeError("ref_swifttd_example_run failed")
    return fields, v


# ---------------------------------------------------------------------------
# Backward pass and the example networks (mlp-xor: Topological; iPC: Pipeline)
# ---------------------------------------------------------------------------
def backward(from_id, to_id, w, dval, n_units, lo, hi, apply=0, value=None, out=None,
             descending=True, dead=None):
    """DoBackwardPass over the given connections (Pipeline order when
    descending, else one Topological level range). Returns out (n_units
    float32; entries [lo, hi) written)."""
    out = np.zeros(n_units, np.float32) if out is None else out
    acc = np.zeros(n_units, np.float32)
    value = None if value is None else np.ascontiguousarray(value, np.float32)
    orc().oracle_backward(from_id.size, _p(from_id), _p(to_id), _p(dead), _p(w),
                          _p(np.ascontiguousarray(dval, np.float32)), int(descending),
                          n_units, lo, hi, apply, _p(value), _p(out), _p(acc))
    return out


def ipc_value_update(x, eps, bu, gamma, act, mode=1):
    """In place on float32 arrays of equal length."""
    orc().oracle_ipc_value_update(x.size, _p(x), _p(eps), _p(bu), gamma, _p(act), mode)


def mse_sigmoid_grad(act, target):
    act = np.ascontiguousarray(act, np.float32)
    g = np.empty_like(act)
    orc().oracle_mse_sigmoid_grad(act.size, _p(act), _p(np.ascontiguousarray(target, np.float32)),
                                  _p(g))
    return g


class MlpTopo:
    """A layered sigmoid MLP in the reference's Topological mode with the
    mlp_xor.cpp policies: FullyConnected layers (dst-major), levels 0..L.
    layers = unit counts per level; w = weights in connection order."""

    def __init__(self, layers, w, lr=0.5):
        self.layers = list(layers)
        self.begin = np.cumsum([0] + self.layers)
        self.n_units = int(self.begin[-1])
        frm, to, self.level_conn = [], [], [0]
        for L in range(1, len(self.layers)):
            for u in range(self.begin[L], self.begin[L + 1]):
                for s_ in range(self.begin[L - 1], self.begin[L]):
                    frm.append(s_)
                    to.append(u)
            self.level_conn.append(len(frm))
        self.from_id = np.array(frm, np.uint32)
        self.to_id = np.array(to, np.uint32)
        self.w = np.array(w, np.float32, copy=True)
        self.lr = lr
        self.act = np.zeros(self.n_units, np.float32)
        self.grad = np.zeros(self.n_units, np.float32)

    def _conns(self, L):  # connections with SrcLevel == L
        return slice(self.level_conn[L], self.level_conn[L + 1])

    def forward(self, x):
        self.act[:self.layers[0]] = x
        acc = np.zeros(self.n_units, np.float32)
        for L in range(1, len(self.layers)):
            c = self._conns(L - 1)
            f, t = np.ascontiguousarray(self.from_id[c]), np.ascontiguousarray(self.to_id[c])
            ww = np.ascontiguousarray(self.w[c])
            orc().oracle_forward_pipeline(f.size, _p(f), _p(t), None, _p(ww), _p(self.act),
                                          int(self.begin[L + 1]), int(self.begin[L]), 1, None,
                                          None, _p(acc))
        return self.act[self.begin[-2]:].copy()

    def step(self, x, target):
        """DoStep: forward, MSELoss, backward (levels L..1), gradient update."""
        self.forward(x)
        top = len(self.layers) - 1
        o = slice(self.begin[top], self.begin[top + 1])
        self.grad[o] = mse_sigmoid_grad(self.act[o], np.atleast_1d(target))
        for L in range(top - 1, 0, -1):
            c = self._conns(L)
            self.grad = backward(np.ascontiguousarray(self.from_id[c]),
                                 np.ascontiguousarray(self.to_id[c]),
                                 np.ascontiguousarray(self.w[c]), self.grad, self.n_units,
                                 int(self.begin[L]), int(self.begin[L + 1]), apply=4,
                                 value=self.act, out=self.grad, descending=False)
        self.w = update_post(self.from_id, self.to_id, self.act, self.grad, self.w, 1, self.lr)


def ipc_prestep(x, inputs, hidden):
    """Activation = f(ValueNode): inputs as given (DoForwardPass clamps them),
    tanh for hidden units, identity for the rest (ipc_multilayer.cpp:220-228)."""
    lo, hi = hidden
    act = np.array(x, np.float32, copy=True)
    act[:inputs.size] = inputs
    ipc_value_update(x[lo:hi].copy(), np.zeros(hi - lo, np.float32),
                     np.zeros(hi - lo, np.float32), 0.0, act[lo:hi], mode=0)
    return act


def ipc_forward(from_id, to_id, w, act, x, n_in):
    """DoForwardPass, Pipeline, iPC Apply: eps = x - mu for units >= n_in."""
    n = x.size
    err = np.zeros(n, np.float32)
    acc = np.zeros(n, np.float32)
    act = np.array(act, np.float32, copy=True)
    orc().oracle_forward_pipeline(from_id.size, _p(from_id), _p(to_id), None, _p(w), _p(act),
                                  n, n_in, 3, _p(x), _p(err), _p(acc))
    return err


def ipc_backward(from_id, to_id, w, err, x, hidden):
    """DoBackwardPass, Pipeline: BottomUp of the hidden units."""
    lo, hi = hidden
    return backward(from_id, to_id, w, err, x.size, lo, hi, apply=5, value=x,
                    descending=True)


def ipc_hidden_update(x, err, bu, act, gamma, hidden):
    """Value-node update of the hidden units and the next pre-step, in place
    on x and act (ipc_multilayer.cpp:239-245)."""
    lo, hi = hidden
    xh, eh, bh, ah = x[lo:hi].copy(), err[lo:hi].copy(), bu[lo:hi].copy(), act[lo:hi].copy()
    ipc_value_update(xh, eh, bh, gamma, ah, mode=1)
    x[lo:hi] = xh
    act[lo:hi] = ah


def ipc_step(from_id, to_id, w, x, inputs, hidden, gamma, alpha):
    """The iPC example's iPCStep (ipc_multilayer.cpp:214-246) on a Pipeline
    network: units [0, n_in) inputs, `hidden` = (lo, hi) tanh units, the rest
    identity outputs. In place on w and x; returns (err, act)."""
    act = ipc_prestep(x, inputs, hidden)
    err = ipc_forward(from_id, to_id, w, act, x, inputs.size)
    bu = ipc_backward(from_id, to_id, w, err, x, hidden)
    w[:] = update_post(from_id, to_id, act, err, w, 2, alpha)
    ipc_hidden_update(x, err, bu, act, gamma, hidden)
    return err, act


def ref_mlp_run(n_in, n_hidden, seed, epochs, inputs, targets):
    L = ref()
    if L is None:
        raise FileNotFoundError(f"{REF_SO} was not built")
    inputs = np.ascontiguousarray(inputs, np.float32)
    targets = np.ascontiguousarray(targets, np.float32)
    maxc = n_in * n_hidden + n_hidden + 16
    w0, w1 = np.zeros(maxc, np.float32), np.zeros(maxc, np.float32)
    preds = np.zeros(targets.size, np.float32)
    m = L.ref_mlp_run(n_in, n_hidden, seed, epochs, targets.size, _p(inputs), _p(targets),
                      _p(w0), _p(w1), _p(preds), maxc)
    if m < 0:
        raise RuntimeError("ref_mlp_run failed")
    return w0[:m], w1[:m], preds


def ref_ipc_run(inputs, targets, w, x):
    """The example's own iPCStep for len(targets) steps (3 -> 16 -> 1)."""
    L = ref()
    if L is None:
        raise FileNotFoundError(f"{REF_SO} was not built")
    w = np.array(w, np.float32, copy=True)
    x = np.array(x, np.float32, copy=True)
    err = np.zeros_like(x)
    inputs = np.ascontiguousarray(inputs, np.float32)
    targets = np.ascontiguousarray(targets, np.float32)
    m = L.ref_ipc_run(targets.size, _p(inputs), _p(targets), _p(w), _p(x), _p(err), w.size)
    if m != w.size:
        raise RuntimeError("ref_ipc_run failed")
    return w, x, err


# ---------------------------------------------------------------------------
# Unit levels (RecomputeLevels, plastix.hpp:466-537)
# ---------------------------------------------------------------------------
def recompute_levels(n_units, n_input, from_id, to_id, dead=None, level=None):
    """Returns (levels uint16[n_units], rounds). ``level`` gives the levels
    before the call (input units keep theirs unless re-reached); zeros if
    omitted."""
    lv = np.zeros(n_units, np.uint16) if level is None else np.array(level, np.uint16)
    f = np.ascontiguousarray(from_id, np.uint32)
    t = np.ascontiguousarray(to_id, np.uint32)
    d = None if dead is None else np.ascontiguousarray(dead, np.uint8)
    r = orc().oracle_recompute_levels(n_units, n_input, f.size, _p(f), _p(t), _p(d), _p(lv))
    if r < 0:
        raise ValueError("connection names a unit outside [0, n_units)")
    return lv, int(r)


def sort_connections_by_level(n_units, n_input, from_id, to_id, dead=None, level=None):
    """SortConnectionsByLevel (plastix.hpp:539-579): (levels, perm, sorted
    SrcLevel, NumLevels); perm is the stable order by SrcLevel."""
    lv, _ = recompute_levels(n_units, n_input, from_id, to_id, dead, level)
    f = np.ascontiguousarray(from_id, np.uint32)
    src_level = lv[f] if f.size else np.zeros(0, np.uint16)
    perm = stable_sort_perm_u32(src_level.astype(np.uint32))
    sorted_level = src_level[perm.astype(np.int64)] if f.size else src_level
    num_levels = int(sorted_level[-1]) + 1 if f.size else 0
    return lv, perm, sorted_level, num_levels


def ref_levels_run(n_units, n_input, from_id, to_id, dead=None):
    """The reference itself: a Topological Network built with these units and
    connections (its constructor runs SortConnectionsByLevel). Returns
    (levels, FromId, ToId, SrcLevel, Dead after the sort) or None when the
    reference was not built here."""
    R = ref()
    if R is None:
        return None
    n = len(from_id)
    f = np.ascontiguousarray(from_id, np.uint32)
    t = np.ascontiguousarray(to_id, np.uint32)
    d = None if dead is None else np.ascontiguousarray(dead, np.uint8)
    lv = np.zeros(n_units, np.uint16)
    fo, to_, so = (np.zeros(n, np.uint32), np.zeros(n, np.uint32), np.zeros(n, np.uint16))
    do = np.zeros(n, np.uint8)
    rc = R.ref_levels_run(n_units, n_input, n, _p(f), _p(t), _p(d), _p(lv), _p(fo), _p(to_),
                          _p(so), _p(do))
    if rc != 0:
        raise RuntimeError(f"ref_levels_run failed ({rc})")
    return lv, fo, to_, so, do


# ---------------------------------------------------------------------------
# Structural policies through the reference's Network (oracle/structural_policies.hpp)
# ---------------------------------------------------------------------------
STRUCTURAL_CASES = {  # name: (variant, n_in, h1, h2, seed, steps, cap)
    "small": (0, 4, 6, 3, 5, 5, 4096),
    "medium": (1, 32, 200, 50, 9, 3, 200_000),
}


def structural_inputs(name):
    variant, n_in, h1, h2, seed, steps, cap = STRUCTURAL_CASES[name]
    return np.random.default_rng(100 + seed).uniform(-1, 1, (steps, n_in)).astype(np.float32)


def ref_structural_run(name):
    """A Topological reference network n_in -> FC h1 -> FC h2 stepped with the
    structural test policies; returns a dict of the per-step outputs, the final
    connections (storage order) and the units' levels and activations, or None
    when the reference was not built here."""
    R = ref()
    if R is None:
        return None
    variant, n_in, h1, h2, seed, steps, cap = STRUCTURAL_CASES[name]
    x = structural_inputs(name)
    outs = np.zeros((steps, h2), np.float32)
    frm, to = np.zeros(cap, np.uint32), np.zeros(cap, np.uint32)
    dead, sl = np.zeros(cap, np.uint8), np.zeros(cap, np.uint16)
    w = np.zeros(cap, np.float32)
    nu_cap = n_in + h1 + h2
    level, act = np.zeros(nu_cap, np.uint16), np.zeros(nu_cap, np.float32)
    n_conn, n_units = ctypes.c_uint64(0), ctypes.c_uint64(0)
    rc = R.ref_structural_run(variant, n_in, h1, h2, seed, steps, _p(x), cap, _p(outs), _p(frm),
                              _p(to), _p(dead), _p(sl), _p(w), ctypes.byref(n_conn), _p(level),
                              _p(act), ctypes.byref(n_units))
    if rc != 0:
        raise RuntimeError(f"ref_structural_run failed ({rc})")
    m, n = n_conn.value, n_units.value
    return {"outputs": outs, "from": frm[:m], "to": to[:m], "dead": dead[:m],
            "src_level": sl[:m], "w": w[:m], "level": level[:n], "act": act[:n]}
