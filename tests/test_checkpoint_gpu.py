"""Checkpoint / resume of the device runtime: each stateful layer is stepped,
saved, stepped further; a second instance built the same way is loaded from
the file and stepped the same way; every state tensor must match bit for bit
(and the host reads nothing but the file)."""
import numpy as np
import pytest
import torch

from plastix_b200 import workloads
from plastix_b200.runtime import (HebbianSweepLayer, PredictiveCodingNet, StructuralLayer,
                                  SwiftTDLearner)

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def check_resume(tmp_path, make, run, state):
    a = make()
    run(a, 0, 3)
    a.save(tmp_path / "ckpt.npz")
    run(a, 3, 3)
    b = make()
    b.load(tmp_path / "ckpt.npz")
    run(b, 3, 3)
    torch.cuda.synchronize()
    for (k, x), (_, y) in zip(state(a).items(), state(b).items()):
        np.testing.assert_array_equal(bits(y), bits(x), err_msg=k)


def test_hebbian_sweep_layer_resumes(ctx, tmp_path):
    L = workloads.sparse_layer(5000, 3000, 200_000, seed=4)
    i32 = lambda a: torch.from_numpy(a.view(np.int32)).cuda()  # noqa: E731
    act = torch.from_numpy(L.act_in).cuda()
    make = lambda: HebbianSweepLayer(ctx, L.n_src, L.n_dst, i32(L.from_id), i32(L.to_id),  # noqa
                                     torch.from_numpy(L.weight).cuda())
    check_resume(tmp_path, make, lambda m, s0, k: [m.step(act) for _ in range(k)],
                 lambda m: {"w": m.weight, "e": m.trace, "a": m.act_dst})


def test_structural_layer_resumes(ctx, tmp_path):
    g = torch.Generator(device="cuda").manual_seed(3)
    n_src, n_dst, n = 20_000, 20_000, 300_000
    f = torch.randint(0, n_src, (n,), generator=g, device="cuda", dtype=torch.int32)
    t = torch.sort(torch.randint(n_src, n_src + n_dst, (n,), generator=g, device="cuda",
                                 dtype=torch.int32)).values
    w = torch.randn(n, generator=g, device="cuda") * 0.1
    age = torch.zeros(n, dtype=torch.uint8, device="cuda")
    act = torch.rand(n_src, generator=g, device="cuda")
    make = lambda: StructuralLayer(ctx, n_src, n_dst, f, t, w, age, threshold=0.02, seed=5)  # noqa
    check_resume(tmp_path, make, lambda m, s0, k: [m.step(act) for _ in range(k)],
                 lambda m: {"f": m.f, "t": m.t, "w": m.w, "age": m.age, "a": m.act_dst})


def test_swifttd_learner_resumes(ctx, tmp_path):
    n = 50_000
    rng = np.random.default_rng(2)
    sets = [torch.from_numpy(np.sort(rng.choice(n, 300, replace=False)).astype(np.int32)).cuda()
            for _ in range(6)]
    rw = torch.from_numpy(rng.normal(size=6).astype(np.float32)).cuda()
    make = lambda: SwiftTDLearner(ctx, n, max_active=300)  # noqa: E731
    check_resume(tmp_path, make,
                 lambda m, s0, k: [m.step(sets[s0 + i], rw[s0 + i:s0 + i + 1]) for i in range(k)],
                 lambda m: {"state": m.state, "globals": m.globals, "v": m.v})


@pytest.mark.parametrize("layout", ["csr", "chunked"])
def test_predictive_coding_net_resumes(ctx, tmp_path, layout):
    size, fan_in = 4000, 64
    layers = [size] * 4
    begin = np.concatenate([[0], np.cumsum(layers)])
    rng = np.random.default_rng(8)
    blocks = []
    for l in range(3):
        to = np.repeat(np.arange(size, dtype=np.uint32) + np.uint32(begin[l + 1]), fan_in)
        frm = (rng.integers(0, size, to.size) + begin[l]).astype(np.uint32)
        w = rng.normal(0, 1 / np.sqrt(fan_in), to.size).astype(np.float32)
        blocks.append(tuple(torch.from_numpy(np.ascontiguousarray(a).view(
            np.int32 if a.dtype == np.uint32 else a.dtype)).cuda() for a in (frm, to, w)))
    xs = torch.from_numpy(rng.uniform(0, 1, (6, size)).astype(np.float32)).cuda()
    ts = torch.from_numpy(rng.uniform(-1, 1, (6, size)).astype(np.float32)).cuda()
    make = lambda: PredictiveCodingNet(ctx, layers, blocks, gamma=0.1, alpha=0.005,  # noqa
                                       layout=layout)

    def run(m, s0, k):  # per sample: clamp, 3 inference iterations, weight update
        for i in range(k):
            m.clamp(xs[s0 + i], ts[s0 + i])
            for _ in range(3):
                m.iteration()
            m.update()

    check_resume(tmp_path, make, run, lambda m: m._state_tensors())
