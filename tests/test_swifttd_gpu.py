"""SwiftTD on the device (plx_swifttd_step) against the oracle.

The oracle restatement is pinned bit for bit to the reference's own
examples/swifttd/swifttd.cpp network (test_oracle_pins.py). The device sums V,
Tau, B and VDelta as fixed-order double-precision trees, so it is compared
with the oracle's double-sum form (same per-feature float arithmetic, same
sums rounded once) and, more loosely, with the reference's sequential float
sums. Tolerances: relative 1e-5 on every field and on V, with an absolute
floor of 1e-6 for values that cancel to near zero (weights start at zero).
"""
import numpy as np
import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import SwiftTDLearner

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def active_sets(n, k, steps, seed):
    rng = np.random.default_rng(seed)
    return [np.sort(rng.choice(n, k, replace=False)).astype(np.uint32) for _ in range(steps)]


def dense(n, idx, val=None):
    f = np.zeros(n, np.float32)
    f[idx] = 1.0 if val is None else val
    return f


def run_both(ctx, orc, n, sets, rewards, gamma=0.99, vals=None, acc_f64=True):
    td = SwiftTDLearner(ctx, n, gamma=gamma, max_active=max(1, max(len(s) for s in sets)))
    fields = orc.td_fields(n)
    g = orc.td_globals(gamma=gamma)
    rw = torch.from_numpy(rewards).cuda()
    vs_dev, vs_orc = [], []
    for s, idx in enumerate(sets):
        val = None if vals is None else vals[s]
        idx_d = torch.from_numpy(idx.view(np.int32)).cuda()
        val_d = None if val is None else torch.from_numpy(val).cuda()
        vs_dev.append(td.step(idx_d, rw[s:s + 1], val_d).clone())
        vs_orc.append(orc.swifttd_step(fields, dense(n, idx, val), rewards[s], g, acc_f64))
    ctx.sync()
    v_dev = torch.cat(vs_dev).cpu().numpy()
    return td, fields, g, v_dev, np.array(vs_orc, np.float32)


def check(td, fields, g, v_dev, v_orc, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(v_dev, v_orc, rtol=rtol, atol=atol)
    got = td.fields().cpu().numpy()
    for j in range(10):
        np.testing.assert_allclose(got[j], fields[j], rtol=rtol, atol=atol,
                                   err_msg=f"field {j}")
    gd = td.globals.cpu().numpy()
    np.testing.assert_allclose(gd, g, rtol=rtol, atol=atol)


@pytest.mark.parametrize("n,k", [(65_536, 655), (3_001, 1), (1_027, 1024), (5_000, 1023),
                                 (70_001, 1025), (4_096, 0)])
def test_swifttd_matches_oracle(ctx, orc, n, k):
    steps = 30
    rng = np.random.default_rng(n + k)
    sets = active_sets(n, k, steps, seed=n)
    rewards = rng.normal(size=steps).astype(np.float32)
    check(*run_both(ctx, orc, n, sets, rewards))


def test_swifttd_both_branches_against_reference_fixture(ctx, orc):
    """The reference-made fixture (Gamma 1.0, 0-5 active features a step, so
    Tau crosses Eta both ways): the device run against the reference's own
    float results, at the same 1e-5 relative bar."""
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / "swifttd_small.npz")
    feats, rewards = z["features"], z["rewards"]
    sets = [np.flatnonzero(f).astype(np.uint32) for f in feats]
    td, fields, g, v_dev, v_orc = run_both(ctx, orc, int(z["n"]), sets, rewards, gamma=1.0,
                                           acc_f64=False)
    np.testing.assert_array_equal(v_orc.view(np.uint32), z["v"].view(np.uint32))
    np.testing.assert_allclose(v_dev, z["v"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(td.fields().cpu().numpy(), z["fields"], rtol=RTOL, atol=ATOL)


def test_swifttd_real_valued_features(ctx, orc):
    n, k, steps = 20_000, 150, 12
    sets = active_sets(n, k, steps, seed=3)
    rng = np.random.default_rng(4)
    vals = [rng.uniform(0.1, 2.0, k).astype(np.float32) for _ in range(steps)]
    rewards = rng.normal(size=steps).astype(np.float32)
    check(*run_both(ctx, orc, n, sets, rewards, vals=vals))


def test_swifttd_close_to_sequential_float_sums(ctx, orc):
    n, k, steps = 65_536, 655, 20
    sets = active_sets(n, k, steps, seed=9)
    rewards = np.random.default_rng(10).normal(size=steps).astype(np.float32)
    check(*run_both(ctx, orc, n, sets, rewards, acc_f64=False), rtol=1e-4, atol=1e-5)


def test_swifttd_rejects_unsorted_active_list(ctx):
    td = SwiftTDLearner(ctx, 10_000, max_active=8)
    idx = torch.tensor([5, 3, 9], dtype=torch.int32, device="cuda")
    td.step(idx, torch.zeros(1, device="cuda"))
    with pytest.raises(_abi.PlxError):
        ctx.sync()
    idx = torch.tensor([5, 10_000], dtype=torch.int32, device="cuda")
    td.step(idx, torch.zeros(1, device="cuda"))
    with pytest.raises(_abi.PlxError):
        ctx.sync()


def test_swifttd_full_size(ctx, orc):
    """4,194,304 features, 20,971 active a step (0.5 %), gamma 0.99: a few
    steps against the oracle's double-sum form."""
    n, k, steps = 1 << 22, 20_971, 4
    sets = active_sets(n, k, steps, seed=17)
    rewards = np.random.default_rng(18).normal(size=steps).astype(np.float32)
    check(*run_both(ctx, orc, n, sets, rewards))


def test_swifttd_step_parts_equal_step(ctx):
    """plx_swifttd_reduce + plx_swifttd_apply give the same bits as
    plx_swifttd_step."""
    n, k, steps = 50_000, 400, 6
    sets = active_sets(n, k, steps, seed=30)
    rw = torch.from_numpy(np.random.default_rng(31).normal(size=steps).astype(np.float32)).cuda()
    a = SwiftTDLearner(ctx, n, max_active=k)
    b = SwiftTDLearner(ctx, n, max_active=k)
    for s, idx in enumerate(sets):
        idx_d = torch.from_numpy(idx.view(np.int32)).cuda()
        a.step(idx_d, rw[s:s + 1])
        b.step_parts(idx_d, rw[s:s + 1])
    ctx.sync()
    np.testing.assert_array_equal(a.fields().cpu().numpy().view(np.uint32),
                                  b.fields().cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(a.globals.cpu().numpy().view(np.uint32),
                                  b.globals.cpu().numpy().view(np.uint32))
