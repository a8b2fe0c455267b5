"""The chunked-source layout (plx_chunked_*): the layout itself is integer
work and checked exactly; row sums fold in a fixed chunked order (compared
with the oracle's reference-order sums at 1e-5 relative, absolute floor
1e-5); per-connection updates are checked bit for bit against the CSR update
of the same rule; and the multilayer iPC sample runs on it against the
oracle."""
import numpy as np
import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import ChunkedRows, Context, DstCsr, PredictiveCodingNet, sweep_update

pytestmark = pytest.mark.gpu
CH = _abi.CHUNK_SOURCES


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def host(t):
    return t.detach().cpu().numpy()


def layer(n_src, n_rows, n, seed, src_base=0, row_base=None, outside=0):
    rng = np.random.default_rng(seed)
    row_base = n_src + src_base if row_base is None else row_base
    rows = np.sort(rng.integers(0, n_rows, n)).astype(np.uint32) + np.uint32(row_base)
    src = (rng.integers(0, n_src, n) + src_base).astype(np.uint32)
    if outside:
        src[rng.choice(n, outside, replace=False)] = np.uint32(src_base + n_src + 5)
    w = rng.normal(0, 0.05, n).astype(np.float32)
    return src, rows, w


@pytest.mark.parametrize("n_src,n_rows,n,outside", [(1000, 300, 50_000, 0),
                                                    (40_000, 2000, 600_000, 17),
                                                    (CH * 2, 500, 200_000, 0),
                                                    (5, 3, 0, 0)])
def test_chunked_layout_is_exact(ctx, n_src, n_rows, n, outside):
    src_base = 100
    src, rows, w = layer(n_src, n_rows, n, seed=n_src + n, src_base=src_base, outside=outside)
    empty = torch.zeros(1, dtype=torch.int32, device="cuda")[:0]
    L = ChunkedRows(ctx, dev(src) if n else empty, dev(rows) if n else empty,
                    dev(w) if n else torch.zeros(1, device="cuda")[:0], src_base, n_src,
                    src_base + n_src, n_rows)
    ctx.sync()
    n_chunks = (n_src + CH - 1) // CH
    seg = host(L.seg_ptr).view(np.uint32).astype(np.int64)
    perm = host(L.perm).view(np.uint32)
    s16 = host(L.src).view(np.uint16)
    wl = host(L.weight)
    inside = (src.astype(np.int64) - src_base < n_src)
    keys = ((src.astype(np.int64) - src_base) // CH) * n_rows + (rows.astype(np.int64)
                                                                 - src_base - n_src)
    n_keys = n_chunks * n_rows
    assert seg[0] == 0 and np.all(np.diff(seg) % 4 == 0)
    counts = np.bincount(keys[inside], minlength=n_keys) if n else np.zeros(n_keys, np.int64)
    pad = np.diff(seg) - counts
    assert np.all((pad >= 0) & (pad < 4))
    valid = perm != 0xFFFFFFFF
    assert valid.sum() == inside.sum()
    # valid slots in slot order = connections stably sorted by (chunk, row)
    order = np.flatnonzero(inside)
    order = order[np.argsort(keys[order], kind="stable")]
    np.testing.assert_array_equal(perm[valid], order.astype(np.uint32))
    slots = np.flatnonzero(valid)
    k_of = keys[perm[valid].astype(np.int64)]
    assert np.all((seg[k_of] <= slots) & (slots < seg[k_of + 1]))
    np.testing.assert_array_equal(s16[valid],
                                  ((src[order].astype(np.int64) - src_base) % CH))
    assert np.all(s16[:seg[-1]][~valid[:seg[-1]]] == CH)
    np.testing.assert_array_equal(wl[valid].view(np.uint32), w[order].view(np.uint32))
    assert np.all(wl[:seg[-1]][~valid[:seg[-1]]] == 0)


@pytest.mark.parametrize("apply", [_abi.APPLY_IDENTITY, _abi.APPLY_IPC_ERROR,
                                   _abi.APPLY_TANH_GRAD, _abi.APPLY_SIGMOID])
def test_chunked_fold_matches_oracle(ctx, orc, apply):
    n_src, n_rows, n = 50_000, 3000, 3_000_000  # ~1000 connections per row, 4 chunks
    src, rows, w = layer(n_src, n_rows, n, seed=apply)
    act = np.random.default_rng(7).uniform(-1, 1, n_src + n_rows).astype(np.float32)
    value = np.random.default_rng(8).uniform(-1, 1, n_src + n_rows).astype(np.float32)
    L = ChunkedRows(ctx, dev(src), dev(rows), dev(w), 0, n_src, n_src, n_rows)
    out = torch.zeros(n_rows, device="cuda")
    L.fold(dev(act[:n_src]), out, apply, value=dev(value[n_src:]))
    ctx.sync()
    a = act.copy()
    if apply == _abi.APPLY_TANH_GRAD:
        # the backward apply on rows of a float64 sum (row order is irrelevant
        # at this tolerance)
        acc = np.zeros(n_rows, np.float64)
        np.add.at(acc, rows - n_src, w.astype(np.float64) * act[src])
        t = np.tanh(value[n_src:].astype(np.float64))
        want = ((1 - t * t) * acc).astype(np.float32)
    else:
        want_act, err = orc.forward_pipeline(src, rows, w, a, n_src, apply=apply, value=value)
        want = err[n_src:] if apply == _abi.APPLY_IPC_ERROR else want_act[n_src:]
    # ~1000-term sums: the oracle's own sequential float sum carries ~1e-6
    # relative error; the absolute floor covers rows that cancel to near zero
    np.testing.assert_allclose(host(out), want, rtol=1e-5, atol=2e-5)


@pytest.mark.parametrize("n_src,n_rows,n", [(50_000, 3000, 3_000_000), (700, 5, 2000),
                                            (CH * 3 + 1, 1, 40_000)])
def test_fold_with_fused_value_update_equals_separate_calls(ctx, n_src, n_rows, n):
    """The iPC backward fold with the value-node update in its epilogue
    (plx_chunked_fold_ipc_value) leaves x and act equal bit for bit to the
    separate fold (TANH_GRAD into bu) + plx_ipc_value_update (mode 1)."""
    src, rows, w = layer(n_src, n_rows, n, seed=n_rows)
    rng = np.random.default_rng(n)
    err_src = rng.uniform(-1, 1, n_src).astype(np.float32)
    x0 = rng.uniform(-2, 2, n_rows).astype(np.float32)
    eps = rng.uniform(-1, 1, n_rows).astype(np.float32)
    L = ChunkedRows(ctx, dev(src), dev(rows), dev(w), 0, n_src, n_src, n_rows)
    # separate
    x_a, act_a, bu = dev(x0), torch.zeros(n_rows, device="cuda"), torch.zeros(n_rows, device="cuda")
    L.fold(dev(err_src), bu, _abi.APPLY_TANH_GRAD, value=x_a)
    _abi.check(_abi.lib().plx_ipc_value_update(ctx.handle, n_rows, x_a.data_ptr(),
                                               dev(eps).data_ptr(), bu.data_ptr(), 0.1,
                                               act_a.data_ptr(), 1), "plx_ipc_value_update")
    # fused
    x_b, act_b = dev(x0), torch.zeros(n_rows, device="cuda")
    L.fold_ipc_value(dev(err_src), x_b, dev(eps), act_b, 0.1)
    ctx.sync()
    np.testing.assert_array_equal(host(x_b), host(x_a))
    np.testing.assert_array_equal(host(act_b), host(act_a))
    assert np.all(host(bu) == 0)  # the separate update zeroes bu; the fused one never writes it


@pytest.mark.parametrize("kind", [_abi.UPDATE_GRADIENT, _abi.UPDATE_HEBBIAN])
def test_chunked_update_equals_csr_update(ctx, kind):
    n_src, n_rows, n = 40_000, 1500, 1_200_000
    src, rows, w = layer(n_src, n_rows, n, seed=kind)
    rng = np.random.default_rng(kind)
    act = rng.uniform(-1, 1, n_src).astype(np.float32)
    post = rng.normal(size=n_rows).astype(np.float32)
    L = ChunkedRows(ctx, dev(src), dev(rows), dev(w), 0, n_src, n_src, n_rows)
    L.update(dev(act), dev(post), kind, 0.01)
    csr = DstCsr(ctx, dev(rows), n_src, n_rows, use_to_id=False)
    w_csr = dev(w)
    sweep_update(ctx, csr, dev(src), dev(act), dev(post), w_csr, w_csr, kind=kind, rate=0.01)
    ctx.sync()
    np.testing.assert_array_equal(host(L.weights_in_original_order(n)).view(np.uint32),
                                  host(w_csr).view(np.uint32))


def test_chunked_transposed_update_equals_forward_copy(ctx):
    """HEBBIAN_T on the source-major chunked copy gives the same bits as
    HEBBIAN on the destination-major one."""
    n_src, n_rows, n = 30_000, 30_000, 900_000
    src, rows, w = layer(n_src, n_rows, n, seed=5)
    rng = np.random.default_rng(6)
    act = rng.uniform(-1, 1, n_src).astype(np.float32)
    err = rng.normal(size=n_rows).astype(np.float32)
    fwd = ChunkedRows(ctx, dev(src), dev(rows), dev(w), 0, n_src, n_src, n_rows)
    bwd = ChunkedRows(ctx, dev(rows), dev(src), dev(w), n_src, n_rows, 0, n_src)
    fwd.update(dev(act), dev(err), _abi.UPDATE_HEBBIAN, 0.005)
    bwd.update(dev(err), dev(act), _abi.UPDATE_HEBBIAN_T, 0.005)
    ctx.sync()
    np.testing.assert_array_equal(host(fwd.weights_in_original_order(n)).view(np.uint32),
                                  host(bwd.weights_in_original_order(n)).view(np.uint32))


def test_ipc_multilayer_chunked_matches_oracle(ctx, orc):
    size, fan_in = 20_000, 300
    layers = [size] * 5
    begin = np.concatenate([[0], np.cumsum(layers)])
    rng = np.random.default_rng(0)
    blocks_np = []
    for l in range(4):
        to = np.repeat(np.arange(size, dtype=np.uint32) + np.uint32(begin[l + 1]), fan_in)
        frm = (rng.integers(0, size, to.size) + begin[l]).astype(np.uint32)
        w = rng.normal(0, 1 / np.sqrt(fan_in), to.size).astype(np.float32)
        blocks_np.append((frm, to, w))
    net = PredictiveCodingNet(ctx, layers, [tuple(dev(a) for a in b) for b in blocks_np],
                              gamma=0.1, alpha=0.005, layout="chunked")
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
    np.testing.assert_allclose(host(net.err), err, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(net.x), x, rtol=1e-5, atol=1e-5)
    off = 0
    for l in range(4):
        m = blocks_np[l][0].size
        got = host(net.weights(l, m))
        np.testing.assert_allclose(got, w[off:off + m], rtol=1e-5, atol=1e-6)
        if l in net.bwd:
            np.testing.assert_array_equal(
                host(net.bwd[l].weights_in_original_order(m)).view(np.uint32),
                got.view(np.uint32))
        off += m
