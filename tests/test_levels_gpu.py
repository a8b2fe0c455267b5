"""RecomputeLevels / SortConnectionsByLevel on the device (plx_recompute_levels,
plx_src_levels + radix sort + Gather) against the reference's own fixture
and the oracle, bit for bit: levels of every unit, the number of rounds, the
connections' sorted order and SrcLevels."""
from pathlib import Path

import numpy as np
import pytest
import torch

from plastix_b200 import _abi, workloads
from plastix_b200.runtime import recompute_levels, sort_connections_by_level

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).cuda()


def host(t, dtype):
    return t.detach().cpu().numpy().view(dtype)


def run_levels(ctx, n_units, n_input, f, t, d=None, level0=None):
    level = dev(np.zeros(n_units, np.uint16) if level0 is None else level0, np.int16) \
        if n_units else torch.zeros(1, dtype=torch.int16, device="cuda")
    rounds = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    ft = dev(f, np.int32) if len(f) else torch.zeros(1, dtype=torch.int32, device="cuda")[:0]
    tt = dev(t, np.int32) if len(t) else torch.zeros(1, dtype=torch.int32, device="cuda")[:0]
    dt = None if d is None else dev(d, np.uint8)
    recompute_levels(ctx, n_units, n_input, ft, tt, level, dead=dt, rounds=rounds)
    ctx.sync()
    return host(level, np.uint16)[:n_units], int(rounds.item())


def layered_graph(n_input, width, n_layers, fan_in, seed):
    """Every non-input unit takes fan_in connections from units of the 1-3
    layers below it: all units are reached, levels follow the longest path."""
    rng = np.random.default_rng(seed)
    starts = [0, n_input] + [n_input + width * (k + 1) for k in range(n_layers)]
    frm, to = [], []
    for k in range(1, n_layers + 1):
        lo_layer = max(0, k - 3)
        src_lo, src_hi = starts[lo_layer], starts[k]
        dst = np.repeat(np.arange(starts[k], starts[k + 1]), fan_in)
        frm.append(rng.integers(src_lo, src_hi, dst.size))
        to.append(dst)
    f = np.concatenate(frm).astype(np.uint32)
    t = np.concatenate(to).astype(np.uint32)
    order = rng.permutation(f.size)
    return starts[-1], np.ascontiguousarray(f[order]), np.ascontiguousarray(t[order])


@pytest.mark.parametrize("name", ["dag", "cyclic", "dead", "into_inputs"])
def test_level_sort_matches_reference_fixture(ctx, name):
    """The fixture is the reference's Topological constructor output."""
    z = np.load(GOLDEN / "levels_small.npz")
    nu, ni, nc, seed, back, into = (int(x) for x in z[f"{name}_params"])
    f, t, d = workloads.level_graph(nu, ni, nc, seed, back_edges=back,
                                    dead_frac=float(z[f"{name}_dead_frac"]), into_inputs=into)
    level = torch.zeros(nu, dtype=torch.int16, device="cuda")
    fd, td = dev(f, np.int32), dev(t, np.int32)
    f2, t2 = torch.empty_like(fd), torch.empty_like(td)
    pairs = [(fd, f2), (td, t2)]
    dd = None
    if d is not None:
        dd = dev(d, np.uint8)
        d2 = torch.empty_like(dd)
        pairs.append((dd, d2))
    perm, sl, num_levels = sort_connections_by_level(ctx, nu, ni, fd, td, level, pairs, dead=dd)
    ctx.sync()
    np.testing.assert_array_equal(host(level, np.uint16), z[f"{name}_level"])
    np.testing.assert_array_equal(host(f2, np.uint32), z[f"{name}_from"])
    np.testing.assert_array_equal(host(t2, np.uint32), z[f"{name}_to"])
    np.testing.assert_array_equal(host(sl, np.uint16), z[f"{name}_src_level"])
    if d is not None:
        np.testing.assert_array_equal(host(d2, np.uint8), z[f"{name}_dead"])
    assert int(num_levels.item()) == int(z[f"{name}_src_level"].max()) + 1


@pytest.mark.parametrize("width,n_layers,fan_in", [(1000, 12, 4), (20000, 50, 8)])
def test_levels_layered_graph(ctx, orc, width, n_layers, fan_in):
    n_units, f, t = layered_graph(64, width, n_layers, fan_in, seed=width)
    lv, rounds = run_levels(ctx, n_units, 64, f, t)
    want, want_rounds = orc.recompute_levels(n_units, 64, f, t)
    np.testing.assert_array_equal(lv, want)
    assert rounds == want_rounds
    assert lv[64:].min() >= 1  # every unit reached


@pytest.mark.parametrize("back,dead_frac,into", [(0, 0.0, 0), (200, 0.0, 0), (0, 0.2, 0),
                                                 (50, 0.1, 40)])
def test_levels_random_graphs(ctx, orc, back, dead_frac, into):
    nu, ni = 400_000, 500
    f, t, d = workloads.level_graph(nu, ni, 3_000_000, 5 + back + into, back_edges=back,
                                    dead_frac=dead_frac, into_inputs=into)
    lv0 = np.random.default_rng(1).integers(0, 9, nu).astype(np.uint16)  # stale levels
    lv, rounds = run_levels(ctx, nu, ni, f, t, d, level0=lv0)
    want, want_rounds = orc.recompute_levels(nu, ni, f, t, d, level=lv0)
    np.testing.assert_array_equal(lv, want)
    assert rounds == want_rounds


@pytest.mark.parametrize("dead_frac", [0.0, 0.3])
def test_levels_two_level_graph(ctx, orc, dead_frac):
    """The structural configuration's shape (inputs -> destinations): the
    pass ends within its edge-centric rounds, without outgoing lists."""
    rng = np.random.default_rng(21)
    n_in, n_out, n = 300_000, 300_000, 1_500_000
    f = rng.integers(0, n_in, n).astype(np.uint32)
    t = rng.integers(n_in, n_in + n_out, n).astype(np.uint32)
    d = (rng.random(n) < dead_frac).astype(np.uint8) if dead_frac else None
    lv, rounds = run_levels(ctx, n_in + n_out, n_in, f, t, d)
    want, want_rounds = orc.recompute_levels(n_in + n_out, n_in, f, t, d)
    np.testing.assert_array_equal(lv, want)
    assert rounds == want_rounds == 2


def test_levels_deep_chain_wraps_uint16(ctx, orc):
    """70,000 rounds in one launch; levels past 65535 wrap as the reference's
    uint16 cast does."""
    n = 70_001
    f = np.arange(0, n - 1, dtype=np.uint32)
    t = np.arange(1, n, dtype=np.uint32)
    perm = np.random.default_rng(3).permutation(f.size)
    f, t = np.ascontiguousarray(f[perm]), np.ascontiguousarray(t[perm])
    lv, rounds = run_levels(ctx, n, 1, f, t)
    want, want_rounds = orc.recompute_levels(n, 1, f, t)
    np.testing.assert_array_equal(lv, want)
    assert rounds == want_rounds == n
    assert lv[65536] == 0 and lv[65537] == 1


def test_levels_edge_cases(ctx, orc):
    # no connections: only the reset of non-input levels
    lv, r = run_levels(ctx, 5, 2, [], [], level0=np.array([7, 8, 9, 9, 9], np.uint16))
    np.testing.assert_array_equal(lv, [7, 8, 0, 0, 0])
    assert r == 0
    # no input units
    lv, r = run_levels(ctx, 4, 0, np.array([0, 1, 2], np.uint32), np.array([1, 2, 3], np.uint32))
    assert r == 0 and not lv.any()
    # all units are inputs
    lv, r = run_levels(ctx, 3, 3, np.array([0, 1], np.uint32), np.array([1, 2], np.uint32),
                       level0=np.array([4, 4, 4], np.uint16))
    want, wr = orc.recompute_levels(3, 3, [0, 1], [1, 2], level=[4, 4, 4])
    np.testing.assert_array_equal(lv, want)
    assert r == wr
    # an input unit fed by a reached unit gets a level (reference behaviour)
    lv, _ = run_levels(ctx, 3, 1, np.array([0, 1], np.uint32), np.array([1, 0], np.uint32))
    np.testing.assert_array_equal(lv, [2, 1, 0])
    # zero units
    lv, r = run_levels(ctx, 0, 0, [], [])
    assert r == 0


def test_levels_bad_index_reports_arg(ctx):
    level = torch.zeros(4, dtype=torch.int16, device="cuda")
    f = dev(np.array([0, 9], np.uint32), np.int32)
    t = dev(np.array([1, 2], np.uint32), np.int32)
    recompute_levels(ctx, 4, 1, f, t, level)
    with pytest.raises(_abi.PlxError) as e:
        ctx.sync()
    assert e.value.code == _abi.PLX_ERR_ARG
    ctx.sync()  # the status word was consumed; the context stays usable
