"""Pins the oracle restatement: against the reference's own tests' known
answers, the committed golden fixtures (made by the reference itself), and --
where it was built here -- the reference compiled from its sources."""
from pathlib import Path

import numpy as np
import pytest

from plastix_b200 import workloads

GOLDEN = Path(__file__).resolve().parent / "golden"


def fc_edges(layers):
    """Connections of FullyConnected builders in reference order
    (include/plastix/layers.hpp:56-76: dst-major, src-inner)."""
    frm, to = [], []
    begin, size = 0, layers[0]
    nxt = size
    for n in layers[1:]:
        for u in range(nxt, nxt + n):
            for s in range(begin, begin + size):
                frm.append(s)
                to.append(u)
        begin, size = nxt, n
        nxt += n
    return np.array(frm, np.uint32), np.array(to, np.uint32), nxt


def test_forward_identity_known_answer(orc):
    # reference tests/test_plastix.cpp:127-141 (ForwardPassIdentity)
    f, t, n = fc_edges([2, 1])
    act = np.zeros(n, np.float32)
    act[:2] = [3.0, 5.0]
    out, _ = orc.forward_pipeline(f, t, np.ones(f.size, np.float32), act, 2)
    assert out[2] == 8.0 and out[0] == 3.0 and out[1] == 5.0


def test_pipeline_multilayer_known_answer(orc):
    # reference tests/test_plastix_pipeline.cpp:249-267
    f, t, n = fc_edges([2, 2, 1])
    act = np.zeros(n, np.float32)
    act[:2] = 1.0
    w = np.ones(f.size, np.float32)
    act, _ = orc.forward_pipeline(f, t, w, act, 2)
    assert list(act[2:]) == [2.0, 2.0, 0.0]
    act, _ = orc.forward_pipeline(f, t, w, act, 2)
    assert act[4] == 4.0


def test_three_layer_pipeline_known_answer(orc):
    # reference tests/test_plastix_pipeline.cpp:269-283
    f, t, n = fc_edges([3, 2, 2, 1])
    act = np.zeros(n, np.float32)
    act[:3] = 1.0
    w = np.ones(f.size, np.float32)
    outs = []
    for _ in range(3):
        act, _ = orc.forward_pipeline(f, t, w, act, 3)
        outs.append(act[-1])
    assert outs == [0.0, 0.0, 12.0]


def test_gather_known_answer(orc):
    # reference tests/test_alloc.cpp:51-83: Gather applies a permutation
    perm = np.array([3, 1, 2, 0], np.uint64)
    assert list(orc.gather(perm, np.array([0, 10, 20, 30], np.int32))) == [30, 10, 20, 0]


def test_sort_unique_matches_reference_dedup(orc):
    # plastix.hpp:411-432; reference tests/test_plastix.cpp:1112-1127
    bits = np.array([5, 3, 5, 1, 3, 3], np.uint64)
    assert list(orc.sort_unique_u64(bits)) == [1, 3, 5]


def test_stable_sort_is_stable(orc):
    keys = np.array([2, 1, 2, 0, 1, 70000, 0], np.uint32)
    perm = orc.stable_sort_perm_u32(keys)
    assert list(perm) == list(np.argsort(keys, kind="stable"))


def test_golden_sweep_fixture(orc):
    fx = np.load(GOLDEN / "sweep_hebbian_small.npz")
    L = workloads.sparse_layer(int(fx["n_src"]), int(fx["n_dst"]), int(fx["n_edges"]),
                               seed=int(fx["seed"]))
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, L.n_src,
                               float(fx["decay"]), float(fx["rate"]),
                               sweeps=int(fx["sweeps"]))
    np.testing.assert_array_equal(w, fx["w"])
    np.testing.assert_array_equal(e, fx["trace"])
    np.testing.assert_array_equal(a[L.n_src:], fx["act"])


@pytest.mark.parametrize("seed,n_src,n_dst,n_edges", [(1, 64, 32, 500), (2, 1000, 300, 20000)])
def test_oracle_matches_reference_build(orc, seed, n_src, n_dst, n_edges):
    if orc.ref() is None:
        pytest.skip("reference build not present (only built where the reference tree is)")
    L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=seed)
    w_r, e_r, a_r = orc.ref_sweep_run(n_src, n_dst, L.from_id, L.to_id, L.weight,
                                      L.trace, L.act_in, 5, 0.9, 1e-3)
    act = np.concatenate([L.act_in, np.zeros(n_dst, np.float32)])
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, n_src, 0.9,
                               1e-3, sweeps=5)
    np.testing.assert_array_equal(w, w_r)
    np.testing.assert_array_equal(e, e_r)
    np.testing.assert_array_equal(a[n_src:], a_r)


def _swifttd_oracle_run(orc, feats, rewards, gamma, acc_f64=False):
    fields = orc.td_fields(feats.shape[1])
    g = orc.td_globals(gamma=gamma)
    v = [orc.swifttd_step(fields, feats[s], rewards[s], g, acc_f64) for s in range(len(feats))]
    return fields, np.array(v, np.float32), g


def test_swifttd_oracle_matches_reference_fixture(orc):
    """The SwiftTD restatement against the fixture made by the reference's own
    examples/swifttd/swifttd.cpp network (Gamma 1.0 as that file sets it):
    bit for bit, V after every step and all ten fields at the end."""
    z = np.load(GOLDEN / "swifttd_small.npz")
    fields, v, _ = _swifttd_oracle_run(orc, z["features"], z["rewards"], 1.0)
    np.testing.assert_array_equal(v.view(np.uint32), z["v"].view(np.uint32))
    np.testing.assert_array_equal(fields.view(np.uint32), z["fields"].view(np.uint32))
    assert np.count_nonzero(z["fields"][4]) > 0  # H live: the no-reset branch ran last


def test_swifttd_oracle_matches_reference_build(orc):
    if orc.ref() is None:
        pytest.skip("reference not built here")
    rng = np.random.default_rng(21)
    n, steps = 3000, 25
    feats = np.zeros((steps, n), np.float32)
    for s in range(steps):
        feats[s, rng.choice(n, 30, replace=False)] = 1.0
    rewards = rng.normal(size=steps).astype(np.float32)
    want_f, want_v = orc.ref_swifttd_example_run(feats, rewards)
    fields, v, _ = _swifttd_oracle_run(orc, feats, rewards, 1.0)
    np.testing.assert_array_equal(v.view(np.uint32), want_v.view(np.uint32))
    np.testing.assert_array_equal(fields.view(np.uint32), want_f.view(np.uint32))


def test_swifttd_f64_sums_stay_close_to_sequential_f32(orc):
    """The double-precision-sum form of the oracle (what the device reductions
    are compared with) tracks the reference's sequential float sums."""
    z = np.load(GOLDEN / "swifttd_small.npz")
    f32, v32, _ = _swifttd_oracle_run(orc, z["features"], z["rewards"], 1.0)
    f64, v64, _ = _swifttd_oracle_run(orc, z["features"], z["rewards"], 1.0, acc_f64=True)
    np.testing.assert_allclose(v64, v32, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(f64, f32, rtol=1e-5, atol=1e-6)


def test_mlp_xor_oracle_matches_reference_fixture(orc):
    """The Topological MLP restatement (forward per level, MSELoss, backward
    per level, gradient update) against the reference's own mlp_xor.cpp
    policies: bit for bit after 200 epochs of 4 DoSteps."""
    z = np.load(GOLDEN / "mlp_xor_small.npz")
    net = orc.MlpTopo([2, 8, 1], z["w_init"])
    for _ in range(200):
        for s in range(4):
            net.step(z["inputs"][s], z["targets"][s])
    np.testing.assert_array_equal(net.w.view(np.uint32), z["w_200"].view(np.uint32))
    preds = np.array([net.forward(z["inputs"][s])[0] for s in range(4)], np.float32)
    np.testing.assert_array_equal(preds.view(np.uint32), z["preds_200"].view(np.uint32))


def test_mlp_xor_learns_xor_in_reference_fixture():
    z = np.load(GOLDEN / "mlp_xor_small.npz")
    assert np.array_equal(z["preds_5000"] > 0.5, z["targets"] > 0.5)


def test_ipc_oracle_matches_reference_fixture(orc):
    """The iPC restatement (pre-step, forward with eps = x - mu, Pipeline
    backward in descending connection order, Hebbian update, value-node
    update) against 30 steps of the example's own iPCStep, bit for bit."""
    z = np.load(GOLDEN / "ipc_small.npz")
    f, t, _ = fc_edges([3, 16, 1])
    w, x = z["w0"].copy(), z["x0"].copy()
    for s in range(z["targets"].size):
        x[:3] = z["inputs"][s]
        x[-1] = z["targets"][s]
        err, _ = orc.ipc_step(f, t, w, x, z["inputs"][s], (3, 19), 0.1, 0.005)
    np.testing.assert_array_equal(w.view(np.uint32), z["w"].view(np.uint32))
    np.testing.assert_array_equal(x.view(np.uint32), z["x"].view(np.uint32))
    np.testing.assert_array_equal(err.view(np.uint32), z["err"].view(np.uint32))


def test_backward_descending_order_known_answer(orc):
    # The shape of reference tests/test_plastix.cpp:202-226 (BackwardPassBasic:
    # 2 inputs -> 1 output; BackwardAcc of each source collects Weight times
    # the destination's value, and is cleared after Apply). With weights 2 and
    # 3 and destination value 1 the sources' Apply sees 2 and 3.
    f, t, n = fc_edges([2, 1])
    w = np.array([2.0, 3.0], np.float32)
    dval = np.zeros(n, np.float32)
    dval[2] = 1.0
    out = orc.backward(f, t, w, dval, n, 0, 2)
    assert list(out[:2]) == [2.0, 3.0]


# ---------------------------------------------------------------------------
# RecomputeLevels / SortConnectionsByLevel (plastix.hpp:466-579)
# ---------------------------------------------------------------------------
def test_levels_known_answer(orc):
    # reference tests/test_plastix.cpp:949-960 (FCLayerLevelProgression):
    # 2 inputs -> FC 3 -> FC 1 gives levels 0,0,1,1,1,2
    f, t, n = fc_edges([2, 3, 1])
    lv, rounds = orc.recompute_levels(n, 2, f, t)
    np.testing.assert_array_equal(lv, [0, 0, 1, 1, 1, 2])
    assert rounds == 3
    # :962-974 (ConnectionsSortedBySrcLevel): sorted SrcLevel non-decreasing
    _, perm, sl, nl = orc.sort_connections_by_level(n, 2, f, t)
    assert np.all(np.diff(sl.astype(np.int64)) >= 0) and nl == 2


def _level_case(z, name):
    nu, ni, nc, seed, back, into = (int(x) for x in z[f"{name}_params"])
    return nu, ni, workloads.level_graph(nu, ni, nc, seed, back_edges=back,
                                         dead_frac=float(z[f"{name}_dead_frac"]),
                                         into_inputs=into)


@pytest.mark.parametrize("name", ["dag", "cyclic", "dead", "into_inputs"])
def test_levels_oracle_matches_reference_fixture(orc, name):
    """The reference's own constructor (SortConnectionsByLevel) made the
    fixture: levels of every unit and the connections in sorted order."""
    z = np.load(GOLDEN / "levels_small.npz")
    nu, ni, (f, t, d) = _level_case(z, name)
    lv, perm, sl, _ = orc.sort_connections_by_level(nu, ni, f, t, d)
    np.testing.assert_array_equal(lv, z[f"{name}_level"])
    p = perm.astype(np.int64)
    np.testing.assert_array_equal(f[p], z[f"{name}_from"])
    np.testing.assert_array_equal(t[p], z[f"{name}_to"])
    np.testing.assert_array_equal(sl, z[f"{name}_src_level"])
    if d is not None:
        np.testing.assert_array_equal(d[p], z[f"{name}_dead"])


@pytest.mark.parametrize("seed", [11, 12])
def test_levels_oracle_matches_reference_build(orc, seed):
    if orc.ref() is None:
        pytest.skip("reference build not present")
    rng = np.random.default_rng(seed)
    nu, ni = int(rng.integers(200, 4000)), int(rng.integers(0, 60))
    f, t, d = workloads.level_graph(nu, ni, int(rng.integers(0, 20000)), seed,
                                    back_edges=int(rng.integers(0, 20)), dead_frac=0.1,
                                    into_inputs=int(rng.integers(0, 10)) if ni else 0)
    lv_r, f_r, t_r, sl_r, d_r = orc.ref_levels_run(nu, ni, f, t, d)
    lv, perm, sl, _ = orc.sort_connections_by_level(nu, ni, f, t, d)
    np.testing.assert_array_equal(lv, lv_r)
    np.testing.assert_array_equal(f[perm.astype(np.int64)], f_r)
    np.testing.assert_array_equal(sl, sl_r)


def test_levels_edge_cases(orc):
    # no connections: only the reset of non-input levels (plastix.hpp:470-474)
    lv, r = orc.recompute_levels(5, 2, [], [], level=[7, 8, 9, 9, 9])
    np.testing.assert_array_equal(lv, [7, 8, 0, 0, 0])
    assert r == 0
    # no input units: frontier 0 is empty, every level 0
    lv, r = orc.recompute_levels(4, 0, [0, 1, 2], [1, 2, 3])
    assert r == 0 and not lv.any()
    # a cycle and everything below it stays at 0
    lv, _ = orc.recompute_levels(5, 1, [0, 1, 2, 1], [1, 2, 1, 4])
    np.testing.assert_array_equal(lv, [0, 0, 0, 0, 0])
    # an input unit fed by a reached unit is reached again and gets a level
    lv, _ = orc.recompute_levels(3, 1, [0, 1], [1, 0])
    np.testing.assert_array_equal(lv, [2, 1, 0])
