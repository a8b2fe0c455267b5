"""K1 parity: the sm_100a sweeps against the oracle on the same seeded inputs.

Bit-exact where the reference order is reproduced (rows of up to
PLX_SEQ_ROW_MAX connections, identity/IPC Apply, all per-connection updates);
rtol 1e-5 (atol 1e-6) where the device uses a different but deterministic
reduction order (longer rows) or CUDA's expf/tanhf (sigmoid/tanh Apply).
"""
import numpy as np
import pytest
import torch

from plastix_b200 import _abi, workloads
from plastix_b200.runtime import (DstCsr, HebbianSweepLayer, sweep_forward,
                                  sweep_update)

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ids(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def assert_rows(got, want, row_len, exact_ok=True):
    """Rows of at most PLX_SEQ_ROW_MAX connections: bit-exact (same order as
    the reference); longer rows: within rtol 1e-5 / atol 1e-6."""
    row_len = np.asarray(row_len)
    short = row_len <= _abi.SEQ_ROW_MAX
    if exact_ok:
        np.testing.assert_array_equal(got[short], want[short])
    else:
        np.testing.assert_allclose(got[short], want[short], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got[~short], want[~short], rtol=RTOL, atol=ATOL)


def run_hebbian(ctx, L, sweeps, decay=0.9, rate=1e-3, dead=None, fast=True, layout="csr"):
    layer = HebbianSweepLayer(ctx, L.n_src, L.n_dst, ids(L.from_id), ids(L.to_id),
                              dev(L.weight), dev(L.trace), decay=decay, rate=rate,
                              dead=None if dead is None else dev(dead), fast=fast,
                              layout=layout)
    act = dev(L.act_in)
    for _ in range(sweeps):
        out = layer.step(act)
    ctx.sync()
    return host(layer.weight), host(layer.trace), host(out)


def oracle_hebbian(orc, L, sweeps, decay=0.9, rate=1e-3, dead=None):
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, L.n_src,
                               decay, rate, sweeps=sweeps, dead=dead)
    return w, e, a[L.n_src:]


@pytest.mark.parametrize("n_src,n_dst,n_edges,seed", [
    (1000, 200, 12345, 1),        # ragged tail, several tiles
    (4096, 4096, 2048 * 3, 2),    # exact tile multiple
    (50000, 20000, 300001, 3),    # many tiles, short rows
    (8, 3, 7, 4),                 # fewer edges than one bulk vector
    (1 << 14, 1 << 10, 1 << 16, 5),
])
@pytest.mark.parametrize("fast", [True, False])
def test_fused_hebbian_bit_exact(ctx, orc, n_src, n_dst, n_edges, seed, fast):
    L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=seed)
    got = run_hebbian(ctx, L, sweeps=4, fast=fast)
    want = oracle_hebbian(orc, L, sweeps=4)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


def test_fused_hebbian_golden_fixture(ctx):
    from pathlib import Path
    fx = np.load(Path(__file__).resolve().parent / "golden" / "sweep_hebbian_small.npz")
    L = workloads.sparse_layer(int(fx["n_src"]), int(fx["n_dst"]), int(fx["n_edges"]),
                               seed=int(fx["seed"]))
    w, e, a = run_hebbian(ctx, L, int(fx["sweeps"]), float(fx["decay"]), float(fx["rate"]))
    np.testing.assert_array_equal(w, fx["w"])
    np.testing.assert_array_equal(e, fx["trace"])
    np.testing.assert_array_equal(a, fx["act"])


@pytest.mark.parametrize("fast", [True, False])
def test_fused_hebbian_dead_connections(ctx, orc, fast):
    L = workloads.sparse_layer(3000, 500, 40000, seed=11)
    dead = (np.random.default_rng(3).random(L.from_id.size) < 0.2).astype(np.uint8)
    got = run_hebbian(ctx, L, 3, dead=dead, fast=fast)
    want = oracle_hebbian(orc, L, 3, dead=dead)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


@pytest.mark.parametrize("lens", [
    [256] * 30 + [1, 255, 0, 254, 3] * 20,            # rows at the short-row limit
    [0] * 50 + [7] * 3000 + [0] * 50,                 # empty rows at both stripe ends
    [64, 0, 0, 128, 1] * 4000,                        # many stripes, mixed lengths
    [0, 0, 5, 0, 3000, 0, 1, 2047, 2048, 2049, 0],   # wide + long rows, empty rows
    [257] * 40 + [256] * 40,                          # warp rows vs thread rows
    [10000],                                          # one long row (many tiles)
    [0] * 100,                                        # no connections at all
    [1] * 5000 + [4100] + [3] * 700,                  # long row amid short rows
])
def test_row_shapes(ctx, orc, lens):
    L = workloads.sparse_layer_rows(777, lens, seed=len(lens))
    got = run_hebbian(ctx, L, 2)
    want = oracle_hebbian(orc, L, 2)
    exact = max(lens) <= _abi.SEQ_ROW_MAX
    for g, w in zip(got, want):
        if exact:
            np.testing.assert_array_equal(g, w)
        else:
            np.testing.assert_allclose(g, w, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("apply", [_abi.APPLY_IDENTITY, _abi.APPLY_SIGMOID,
                                   _abi.APPLY_TANH, _abi.APPLY_IPC_ERROR])
@pytest.mark.parametrize("with_dead", [False, True])
@pytest.mark.parametrize("max_len", [300, 257])
def test_forward_apply_kinds(ctx, orc, apply, with_dead, max_len):
    L = workloads.sparse_layer_rows(5000, list(np.random.default_rng(9).integers(0, max_len, 900)),
                                    seed=21)
    dead = (np.random.default_rng(4).random(L.from_id.size) < 0.1).astype(np.uint8) \
        if with_dead else None
    value = np.random.default_rng(5).random(L.n_dst, dtype=np.float32)
    csr = DstCsr(ctx, ids(L.to_id), L.n_src, L.n_dst)
    act_src = dev(L.act_in)
    act_dst = torch.zeros(L.n_dst, device="cuda")
    err = torch.zeros(L.n_dst, device="cuda")
    sweep_forward(ctx, csr, ids(L.from_id), dev(L.weight), act_src, act_dst, apply=apply,
                  dead=None if dead is None else dev(dead), value=dev(value), err_out=err)
    ctx.sync()
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    full_value = np.concatenate([np.zeros(L.n_src, np.float32), value])
    want_act, want_err = orc.forward_pipeline(L.from_id, L.to_id, L.weight, act, L.n_src,
                                              apply=apply, dead=dead, value=full_value)
    got = host(err) if apply == _abi.APPLY_IPC_ERROR else host(act_dst)
    want = want_err[L.n_src:] if apply == _abi.APPLY_IPC_ERROR else want_act[L.n_src:]
    row_len = np.bincount(L.to_id - L.n_src, minlength=L.n_dst)
    assert_rows(got, want, row_len,
                exact_ok=apply in (_abi.APPLY_IDENTITY, _abi.APPLY_IPC_ERROR))


@pytest.mark.parametrize("apply", [_abi.APPLY_IDENTITY, _abi.APPLY_IPC_ERROR,
                                   _abi.APPLY_SIGMOID, _abi.APPLY_TANH])
@pytest.mark.parametrize("with_dead", [False, True])
def test_row_per_thread_forward(ctx, orc, apply, with_dead):
    """plx_sweep_forward_rows (one thread per row, row offsets only): a left
    fold in connection order, so identity and iPC-error rows equal the
    oracle bit for bit at every row length (empty, 1, 2, 1000+), the other
    applies within the device transcendental's tolerance."""
    from plastix_b200.runtime import sweep_forward_rows
    lens = [0, 1, 2, 2, 3, 1, 0, 2] * 300 + [1000, 257, 5000]
    L = workloads.sparse_layer_rows(4000, lens, seed=31)
    dead = (np.random.default_rng(8).random(L.from_id.size) < 0.1).astype(np.uint8) \
        if with_dead else None
    value = np.random.default_rng(5).random(L.n_dst, dtype=np.float32)
    row_ptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    act_dst = torch.zeros(L.n_dst, device="cuda")
    err = torch.zeros(L.n_dst, device="cuda")
    sweep_forward_rows(ctx, dev(row_ptr), ids(L.from_id), dev(L.weight), dev(L.act_in), act_dst,
                       apply=apply, dead=None if dead is None else dev(dead), value=dev(value),
                       err_out=err)
    ctx.sync()
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    full_value = np.concatenate([np.zeros(L.n_src, np.float32), value])
    want_act, want_err = orc.forward_pipeline(L.from_id, L.to_id, L.weight, act, L.n_src,
                                              apply=apply, dead=dead, value=full_value)
    got = host(err) if apply == _abi.APPLY_IPC_ERROR else host(act_dst)
    want = want_err[L.n_src:] if apply == _abi.APPLY_IPC_ERROR else want_act[L.n_src:]
    if apply in (_abi.APPLY_IDENTITY, _abi.APPLY_IPC_ERROR):
        np.testing.assert_array_equal(got, want)
    else:
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_row_per_thread_forward_flags_bad_ids(ctx):
    from plastix_b200.runtime import sweep_forward_rows
    row_ptr = dev(np.array([0, 2, 3], np.int32))
    from_id = ids(np.array([0, 7, 1], np.uint32))  # 7 is past the 4 sources
    out = torch.zeros(2, device="cuda")
    sweep_forward_rows(ctx, row_ptr, from_id, dev(np.ones(3, np.float32)),
                       dev(np.arange(4, dtype=np.float32)), out)
    with pytest.raises(RuntimeError):
        ctx.sync()
    np.testing.assert_array_equal(host(out), [0.0, 1.0])  # the bad id read 0


@pytest.mark.parametrize("kind", [_abi.UPDATE_GRADIENT, _abi.UPDATE_HEBBIAN])
def test_update_kinds(ctx, orc, kind):
    L = workloads.sparse_layer_rows(3000, list(np.random.default_rng(2).integers(0, 600, 700)),
                                    seed=8)
    post = np.random.default_rng(6).normal(size=L.n_dst).astype(np.float32)
    csr = DstCsr(ctx, ids(L.to_id), L.n_src, L.n_dst)
    w = dev(L.weight)
    sweep_update(ctx, csr, ids(L.from_id), dev(L.act_in), dev(post), w, w, kind=kind,
                 rate=0.5)
    ctx.sync()
    full_post = np.concatenate([np.zeros(L.n_src, np.float32), post])
    want = orc.update_post(L.from_id, L.to_id, L.act_in, full_post, L.weight, kind, 0.5)
    np.testing.assert_array_equal(host(w), want)


def test_pipeline_multilayer_known_answer(ctx):
    # reference tests/test_plastix_pipeline.cpp:249-267, all rows in one sweep:
    # 2 inputs -> 2 hidden -> 1 output, weights 1, Pipeline (snapshot) semantics.
    frm = np.array([0, 1, 0, 1, 2, 3], np.uint32)
    to = np.array([2, 2, 3, 3, 4, 4], np.uint32)
    csr = DstCsr(ctx, ids(to), 2, 3)
    act = torch.tensor([1.0, 1.0, 0.0, 0.0, 0.0], device="cuda")
    w = torch.ones(6, device="cuda")
    for expect in ([2.0, 2.0, 0.0], [2.0, 2.0, 4.0]):
        snapshot = act.clone()
        sweep_forward(ctx, csr, ids(frm), w, snapshot, act[2:])
        ctx.sync()
        assert host(act[2:]).tolist() == expect


def test_out_of_range_source_is_reported(ctx):
    frm = np.array([0, 1, 99], np.uint32)
    to = np.array([2, 2, 2], np.uint32)
    csr = DstCsr(ctx, ids(to), 2, 1)
    act = torch.ones(3, device="cuda")
    out = torch.zeros(1, device="cuda")
    sweep_forward(ctx, csr, ids(frm), torch.ones(3, device="cuda"), act, out)
    with pytest.raises(_abi.PlxError) as e:
        ctx.sync()
    assert e.value.code == _abi.PLX_ERR_ARG
    ctx.sync()  # status cleared


def test_invalid_row_ptr_rejected(ctx):
    with pytest.raises(_abi.PlxError):
        DstCsr.from_row_ptr(ctx, torch.tensor([0, 5, 3, 6], dtype=torch.int32))


def test_full_size_sweep_matches_oracle(ctx, orc):
    """The 64M-connection single-layer workload, one fused sweep, compared
    bit for bit with the oracle over the whole layer."""
    n_src = n_dst = 1 << 20
    n = 1 << 26
    from_id, to_id, w, act = workloads.sparse_layer_device(n_src, n_dst, n, 1234, "cuda")
    layer = HebbianSweepLayer(ctx, n_src, n_dst, from_id, to_id, w)
    out = layer.step(act)
    ctx.sync()
    f, t = host(from_id).view(np.uint32), host(to_id).view(np.uint32)
    a_full = np.concatenate([host(act), np.zeros(n_dst, np.float32)])
    ww, ee, aa = orc.step_hebbian(f, t, host(w), np.zeros(n, np.float32), a_full, n_src,
                                  0.9, 1e-3)
    np.testing.assert_array_equal(host(out), aa[n_src:])
    np.testing.assert_array_equal(host(layer.weight), ww)
    np.testing.assert_array_equal(host(layer.trace), ee)


@pytest.mark.parametrize("case", ["dense", "gaps", "outside", "tail", "big", "leading",
                                  "none"])
def test_row_ptr_equals_searchsorted(ctx, case):
    """plx_csr_row_ptr: row_ptr[r] = first connection whose ToId >= row_base + r
    (keys below the range count as before row 0, above it as after the last
    row), row_ptr[n_rows] = n_edges."""
    from ctypes import c_void_p
    from plastix_b200._abi import call
    rng = np.random.default_rng(hash(case) % 1000)
    row_base = 1000
    if case == "dense":
        n_rows, keys = 50_000, rng.integers(0, 50_000, 200_001)
    elif case == "gaps":  # spans wider than one block's staging window
        n_rows = 10_000_000
        keys = np.concatenate([rng.integers(0, 10, 3000), rng.integers(0, n_rows, 5000),
                               rng.integers(n_rows - 10, n_rows, 3000)])
    elif case == "outside":
        n_rows = 3000
        keys = rng.integers(-800, n_rows + 800, 100_003)
    elif case == "tail":
        n_rows, keys = 7, rng.integers(0, 7, 1_026)
    elif case == "leading":  # a million empty rows, then every key in the last rows
        n_rows = 1_000_003
        keys = rng.integers(n_rows - 3, n_rows, 40_000)
    elif case == "none":
        n_rows, keys = 300_000, np.zeros(0, np.int64)
    else:
        n_rows, keys = 1 << 23, rng.integers(0, 1 << 23, 1 << 24)
    to_id = np.sort(keys.astype(np.int64) + row_base).astype(np.uint32)
    t = torch.from_numpy(to_id.view(np.int32)).cuda()
    rp = torch.full((n_rows + 1,), -1, dtype=torch.int32, device="cuda")
    call("plx_csr_row_ptr", ctx.handle, c_void_p(t.data_ptr()), to_id.size, row_base, n_rows,
         c_void_p(rp.data_ptr()))
    ctx.sync()
    want = np.searchsorted(to_id.astype(np.int64), np.arange(n_rows + 1) + row_base,
                           side="left")
    want[-1] = to_id.size
    np.testing.assert_array_equal(rp.cpu().numpy().astype(np.int64), want)


# ---------------------------------------------------------------------------
# The warp-sliced row layout (plx_sweep_forward_hebbian_sliced): one lane per
# row, so every row -- whatever its length -- is folded in the reference's
# order: bit-exact everywhere.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n_src,n_dst,n_edges,seed", [
    (1000, 200, 12345, 1),
    (4096, 4096, 2048 * 3, 2),
    (50000, 20000, 300001, 3),
    (8, 3, 7, 4),
    (1 << 14, 1 << 10, 1 << 16, 5),
    (3000, 513, 40000, 6),        # one row past a 512-row window
])
def test_sliced_hebbian_bit_exact(ctx, orc, n_src, n_dst, n_edges, seed):
    L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=seed)
    got = run_hebbian(ctx, L, sweeps=4, layout="sliced")
    want = oracle_hebbian(orc, L, sweeps=4)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


def test_sliced_hebbian_golden_fixture(ctx):
    from pathlib import Path
    fx = np.load(Path(__file__).resolve().parent / "golden" / "sweep_hebbian_small.npz")
    L = workloads.sparse_layer(int(fx["n_src"]), int(fx["n_dst"]), int(fx["n_edges"]),
                               seed=int(fx["seed"]))
    w, e, a = run_hebbian(ctx, L, int(fx["sweeps"]), float(fx["decay"]), float(fx["rate"]),
                          layout="sliced")
    np.testing.assert_array_equal(w, fx["w"])
    np.testing.assert_array_equal(e, fx["trace"])
    np.testing.assert_array_equal(a, fx["act"])


def test_sliced_hebbian_dead_connections(ctx, orc):
    L = workloads.sparse_layer(3000, 500, 40000, seed=11)
    dead = (np.random.default_rng(3).random(L.from_id.size) < 0.2).astype(np.uint8)
    got = run_hebbian(ctx, L, 3, dead=dead, layout="sliced")
    want = oracle_hebbian(orc, L, 3, dead=dead)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


@pytest.mark.parametrize("lens", [
    [256] * 30 + [1, 255, 0, 254, 3] * 20,
    [0] * 50 + [7] * 3000 + [0] * 50,
    [64, 0, 0, 128, 1] * 4000,
    [0, 0, 5, 0, 3000, 0, 1, 2047, 2048, 2049, 0],   # rows past the staged 96 re-gather
    [257] * 40 + [256] * 40,
    [10000],
    [0] * 100,
    [1] * 5000 + [4100] + [3] * 700,
    [97, 96, 95, 100, 4, 5] * 300,                    # around the staging limit
])
def test_sliced_row_shapes(ctx, orc, lens):
    L = workloads.sparse_layer_rows(777, lens, seed=len(lens))
    got = run_hebbian(ctx, L, 2, layout="sliced")
    want = oracle_hebbian(orc, L, 2)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


def test_sliced_layout_invariants(ctx):
    """perm lists every connection exactly once, in the documented slot
    positions (slot slice_ptr[s] + 128 g + 4 lane + c = connection 4g + c of
    the lane's row), rows sorted by length inside each 512-row window;
    unpack(pack(x)) == x."""
    from plastix_b200.runtime import SlicedRows
    lens = list(np.random.default_rng(1).integers(0, 150, 1300))
    L = workloads.sparse_layer_rows(500, lens, seed=3)
    csr = DstCsr(ctx, ids(L.to_id), L.n_src, L.n_dst)
    sl = SlicedRows(ctx, csr)
    ctx.sync()
    perm = host(sl.perm)[:sl.n_slots].view(np.uint32)
    sp = host(sl.slice_ptr)
    rows = host(sl.lane_row).view(np.uint32)
    ln = host(sl.lane_len)
    rp = host(csr.row_ptr)
    assert sp[0] == 0 and sp[-1] == sl.n_slots and np.all(np.diff(sp) % 128 == 0)
    valid = perm != _abi.SLICED_NONE
    assert np.array_equal(np.sort(perm[valid]), np.arange(L.from_id.size))
    for s in range(sp.size - 1):
        for lane in range(32):
            r = rows[32 * s + lane]
            if r == _abi.SLICED_NONE:
                continue
            assert r // 512 == (32 * s) // 512  # the row belongs to the slice's window
            j = np.arange(ln[32 * s + lane])
            slot = sp[s] + 128 * (j // 4) + 4 * lane + j % 4
            np.testing.assert_array_equal(perm[slot], rp[r] + j)
        lens_s = ln[32 * s:32 * s + 32]
        assert np.all(np.diff(lens_s[rows[32 * s:32 * s + 32] != _abi.SLICED_NONE]) <= 0)
    x = torch.arange(L.from_id.size, dtype=torch.float32, device="cuda")
    np.testing.assert_array_equal(host(sl.unpack(sl.pack(x))), host(x))


def test_sliced_full_size_sweep_matches_oracle(ctx, orc):
    """The 64M-connection single-layer workload in the sliced layout, two
    sweeps, compared bit for bit with the oracle over the whole layer."""
    n_src = n_dst = 1 << 20
    n = 1 << 26
    from_id, to_id, w, act = workloads.sparse_layer_device(n_src, n_dst, n, 1234, "cuda")
    layer = HebbianSweepLayer(ctx, n_src, n_dst, from_id, to_id, w, layout="sliced")
    layer.step(act)
    out = layer.step(act)
    ctx.sync()
    f, t = host(from_id).view(np.uint32), host(to_id).view(np.uint32)
    a_full = np.concatenate([host(act), np.zeros(n_dst, np.float32)])
    ww, ee, aa = orc.step_hebbian(f, t, host(w), np.zeros(n, np.float32), a_full, n_src,
                                  0.9, 1e-3, sweeps=2)
    np.testing.assert_array_equal(host(out), aa[n_src:])
    np.testing.assert_array_equal(host(layer.weight), ww)
    np.testing.assert_array_equal(host(layer.trace), ee)


@pytest.mark.parametrize("n_dst,offset", [(1300, 3), (512, 0), (31, 1001), (4097, 2)])
def test_sliced_hand_off_stores_every_window(ctx, orc, n_dst, offset):
    """The sliced sweep's hand-off: the warp that finishes a 512-row window
    copies it to every peer buffer. Here the peers are three buffers of this
    GPU: after each of three sweeps every buffer holds exactly the layer's
    row values at [offset, offset + n_dst) and nothing else changed, for
    layers whose last window is partial, and with the per-window counters
    reused across sweeps and layers of another size."""
    from ctypes import c_void_p
    lens = list(np.random.default_rng(n_dst).integers(0, 120, n_dst))
    L = workloads.sparse_layer_rows(900, lens, seed=offset)
    layer = HebbianSweepLayer(ctx, L.n_src, L.n_dst, ids(L.from_id), ids(L.to_id),
                              dev(L.weight), dev(L.trace), layout="sliced")
    peer_len = offset + n_dst + 77
    bufs = [torch.full((peer_len,), float("nan"), device="cuda") for _ in range(3)]
    arr = (c_void_p * 3)(*[b.data_ptr() for b in bufs])
    act = dev(L.act_in)
    want_a = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    w_ref, e_ref = L.weight, L.trace
    for _ in range(3):
        for b in bufs:
            b.fill_(float("nan"))
        layer._sliced_sweep(act, arr, 3, offset, peer_len)
        ctx.sync()
        w_ref, e_ref, want_a = orc.step_hebbian(L.from_id, L.to_id, w_ref, e_ref, want_a,
                                                L.n_src, 0.9, 1e-3, sweeps=1)
        out = host(layer.act_dst)
        np.testing.assert_array_equal(out, want_a[L.n_src:])
        for b in bufs:
            hb = host(b)
            np.testing.assert_array_equal(hb[offset:offset + n_dst], out)
            assert np.isnan(hb[:offset]).all() and np.isnan(hb[offset + n_dst:]).all()
