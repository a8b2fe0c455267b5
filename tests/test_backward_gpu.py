"""K2 (backward sweep over a source-major order) and the two example networks
built on it, against the oracle: the XOR MLP (Topological propagation,
sigmoid, MSE, gradient descent) and streaming iPC (Pipeline propagation,
tanh hidden layers, Hebbian update), both pinned to the reference's own
example policies through the golden fixtures.

Exactness: the source-major permutation and row offsets are integer work and
bit-exact. Folds over rows of up to 256 connections are bit-exact against the
oracle; longer rows and anything through expf/tanhf are compared at 1e-5
relative (absolute floor 1e-6 unless stated).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import MlpTopoNet, PredictiveCodingNet, SrcMajor

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def host(t, dtype=None):
    a = t.detach().cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def random_layer(n_src, n_dst, fan_in, seed, src_base=0, dst_base=None, jitter=0):
    """Destination-major connections with fan_in (+- jitter) random sources."""
    rng = np.random.default_rng(seed)
    dst_base = n_src if dst_base is None else dst_base
    counts = fan_in + (rng.integers(-jitter, jitter + 1, n_dst) if jitter else 0)
    counts = np.maximum(counts, 0)
    to = np.repeat(np.arange(n_dst, dtype=np.int64) + dst_base, counts).astype(np.uint32)
    frm = (rng.integers(0, n_src, to.size) + src_base).astype(np.uint32)
    w = rng.normal(0, 1 / np.sqrt(max(fan_in, 1)), to.size).astype(np.float32)
    return frm, to, w


@pytest.mark.parametrize("reverse", [True, False])
@pytest.mark.parametrize("n,n_src,outside", [(0, 5, 0), (1, 1, 0), (70_001, 300, 0),
                                             (200_000, 4096, 1000), (1 << 20, 100_000, 7)])
def test_transpose_is_stable_sort_by_source(ctx, reverse, n, n_src, outside):
    rng = np.random.default_rng(n + n_src)
    base = 1000
    frm = (rng.integers(0, n_src, n) + base).astype(np.uint32)
    if outside and n:
        frm[rng.choice(n, outside, replace=False)] = rng.integers(0, base, outside)
    to = rng.integers(0, 2**31, n).astype(np.uint32)
    w = rng.normal(size=n).astype(np.float32)
    sm = SrcMajor(ctx, dev(frm) if n else torch.zeros(1, dtype=torch.int32, device="cuda")[:0],
                  dev(to) if n else torch.zeros(1, dtype=torch.int32, device="cuda")[:0],
                  dev(w) if n else torch.zeros(1, device="cuda")[:0], base, n_src, reverse)
    ctx.sync()
    key = frm.astype(np.int64) - base
    inside = (key >= 0) & (key < n_src)
    idx = np.flatnonzero(inside)
    order = idx[np.argsort(key[idx], kind="stable")]
    counts = np.bincount(key[idx], minlength=n_src) if n else np.zeros(n_src, np.int64)
    row_ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
    if reverse:
        order = np.concatenate([order[row_ptr[r]:row_ptr[r + 1]][::-1] for r in range(n_src)]
                               + [np.zeros(0, np.int64)])
    np.testing.assert_array_equal(host(sm.csr.row_ptr, np.uint32), row_ptr)
    m = order.size
    assert sm.m == m
    np.testing.assert_array_equal(host(sm.perm, np.uint32)[:m], order.astype(np.uint32))
    np.testing.assert_array_equal(host(sm.to_id, np.uint32)[:m], to[order])
    np.testing.assert_array_equal(host(sm.weight)[:m].view(np.uint32),
                                  w[order].view(np.uint32))


@pytest.mark.parametrize("apply", [_abi.APPLY_IDENTITY, _abi.APPLY_SIGMOID_GRAD,
                                   _abi.APPLY_TANH_GRAD])
@pytest.mark.parametrize("fan_in,jitter,exact", [(40, 20, True), (190, 60, False),
                                                 (3, 3, True)])
def test_backward_sweep_matches_oracle(ctx, orc, apply, fan_in, jitter, exact):
    """DoBackwardPass in Pipeline order (descending connection index) for a
    random layer: sources [0, n_src), destinations after them. Source rows
    have ~fan_in * n_dst / n_src connections: exact when all rows are at
    most 256 long."""
    n_src, n_dst = 3000, 2000
    frm, to, w = random_layer(n_src, n_dst, fan_in, seed=fan_in + apply, jitter=jitter)
    n_units = n_src + n_dst
    rng = np.random.default_rng(apply)
    dval = rng.normal(size=n_units).astype(np.float32)
    value = rng.uniform(-1, 1, n_units).astype(np.float32)
    want = orc.backward(frm, to, w, dval, n_units, 0, n_src, apply=apply, value=value,
                        descending=True)[:n_src]
    sm = SrcMajor(ctx, dev(frm), dev(to), dev(w), 0, n_src, reverse=True)
    out = torch.zeros(n_src, device="cuda")
    sm.backward(dev(dval), out, dev(value[:n_src]), apply)
    ctx.sync()
    longest = int(np.bincount(frm, minlength=n_src).max())
    if exact and apply != _abi.APPLY_TANH_GRAD:
        assert longest <= _abi.SEQ_ROW_MAX
        np.testing.assert_array_equal(host(out).view(np.uint32), want.view(np.uint32))
    else:
        np.testing.assert_allclose(host(out), want, rtol=1e-5, atol=1e-5)


def _mlp_run(ctx, z, epochs):
    net = MlpTopoNet(ctx, [2, 8, 1], z["w_init"], lr=0.5)
    xs = [dev(z["inputs"][s]) for s in range(4)]
    ts = [dev(z["targets"][s:s + 1]) for s in range(4)]
    for _ in range(epochs):
        for s in range(4):
            net.step(xs[s], ts[s])
    preds = np.array([host(net.forward(xs[s]))[0] for s in range(4)], np.float32)
    ctx.sync()
    return host(net.weights()), preds


def test_mlp_xor_200_epochs_matches_reference(ctx):
    z = np.load(GOLDEN / "mlp_xor_small.npz")
    w, preds = _mlp_run(ctx, z, 200)
    np.testing.assert_allclose(w, z["w_200"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(preds, z["preds_200"], rtol=1e-5, atol=1e-6)


def test_mlp_xor_5000_epochs_learns_like_reference(ctx):
    """The C1 configuration: 5,000 epochs of 4 DoSteps, lr 0.5. Over 20,000
    steps the last-bit differences of exp (host libm against the device)
    accumulate, so weights are compared at 1e-5 of the weight vector's scale
    (one weight sits near zero) and predictions at 1e-5 relative."""
    z = np.load(GOLDEN / "mlp_xor_small.npz")
    w, preds = _mlp_run(ctx, z, 5000)
    np.testing.assert_allclose(preds, z["preds_5000"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(w, z["w_5000"], rtol=1e-5,
                               atol=1e-5 * float(np.abs(z["w_5000"]).max()))
    assert np.array_equal(preds > 0.5, z["targets"] > 0.5)


def _fc_blocks(layers):
    begin = np.concatenate([[0], np.cumsum(layers)])
    blocks = []
    for l in range(len(layers) - 1):
        to = np.repeat(np.arange(begin[l + 1], begin[l + 2], dtype=np.uint32), layers[l])
        frm = np.tile(np.arange(begin[l], begin[l + 1], dtype=np.uint32), layers[l + 1])
        blocks.append((frm, to))
    return blocks


def test_ipc_example_shape_matches_reference(ctx):
    """30 iPC steps in the example's order (3 -> 16 -> 1) against the
    reference-made fixture."""
    z = np.load(GOLDEN / "ipc_small.npz")
    blocks = _fc_blocks([3, 16, 1])
    n0 = blocks[0][0].size
    w0 = z["w0"]
    dev_blocks = [(dev(f), dev(t), dev(w0[:n0] if l == 0 else w0[n0:]))
                  for l, (f, t) in enumerate(blocks)]
    net = PredictiveCodingNet(ctx, [3, 16, 1], dev_blocks, gamma=0.1, alpha=0.005)
    net.x.copy_(dev(z["x0"]))
    for s in range(z["targets"].size):
        net.clamp(dev(z["inputs"][s]), dev(z["targets"][s:s + 1]))
        net.example_step()
    ctx.sync()
    w = np.concatenate([host(net.w[0]), host(net.w[1])])
    np.testing.assert_allclose(w, z["w"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(host(net.x), z["x"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(host(net.err), z["err"], rtol=1e-5, atol=1e-6)
    # the source-major copy of the hidden -> output block stays identical
    sm = net.sm[1]
    np.testing.assert_array_equal(host(sm.weight)[:sm.m].view(np.uint32),
                                  host(net.w[1])[host(sm.perm)[:sm.m]].view(np.uint32))


@pytest.mark.parametrize("size,fan_in", [(3000, 100), (2048, 600)])
def test_ipc_multilayer_sample_matches_oracle(ctx, orc, size, fan_in):
    """The multilayer configuration's sample at a reduced size: 5 layers,
    random fan-in, 3 inference iterations then one weight update, against the
    oracle composition of the same reference steps."""
    layers = [size] * 5
    begin = np.concatenate([[0], np.cumsum(layers)])
    blocks_np = [random_layer(layers[l], layers[l + 1], fan_in, seed=l, src_base=begin[l],
                              dst_base=begin[l + 1]) for l in range(4)]
    net = PredictiveCodingNet(ctx, layers, [tuple(dev(a) for a in b) for b in blocks_np],
                              gamma=0.1, alpha=0.005)
    rng = np.random.default_rng(1)
    x0 = rng.uniform(-1, 1, begin[-1]).astype(np.float32)
    inputs = rng.uniform(0, 1, size).astype(np.float32)
    targets = rng.uniform(-1, 1, size).astype(np.float32)
    net.x.copy_(dev(x0))
    net.clamp(dev(inputs), dev(targets))
    for _ in range(3):
        net.iteration()
    net.update()
    ctx.sync()
    frm = np.concatenate([b[0] for b in blocks_np])
    to = np.concatenate([b[1] for b in blocks_np])
    w = np.concatenate([b[2] for b in blocks_np])
    hidden = (int(begin[1]), int(begin[4]))
    x = x0.copy()
    x[:size] = inputs
    x[begin[4]:] = targets
    act = orc.ipc_prestep(x, inputs, hidden)
    for _ in range(3):
        err = orc.ipc_forward(frm, to, w, act, x, size)
        bu = orc.ipc_backward(frm, to, w, err, x, hidden)
        orc.ipc_hidden_update(x, err, bu, act, 0.1, hidden)
    w = orc.update_post(frm, to, act, err, w, 2, 0.005)
    tol = dict(rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(net.err), err, **tol)
    np.testing.assert_allclose(host(net.x), x, **tol)
    got_w = np.concatenate([host(t) for t in net.w])
    np.testing.assert_allclose(got_w, w, rtol=1e-5, atol=1e-6)
    for l, sm in net.sm.items():
        np.testing.assert_array_equal(host(sm.weight)[:sm.m].view(np.uint32),
                                      host(net.w[l])[host(sm.perm)[:sm.m]].view(np.uint32))
