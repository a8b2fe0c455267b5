"""Destination-range sharding, on the CPU: the shard cuts, and two gloo ranks
that each sweep their own rows (with the oracle) and all-gather the
destination slices, against the whole layer swept in one process."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from plastix_b200 import sharding, workloads


def test_balanced_shards_cover_rows_and_balance_edges():
    rng = np.random.default_rng(0)
    counts = rng.integers(0, 50, 1000)
    rp = np.concatenate([[0], np.cumsum(counts)])
    for world in (1, 2, 3, 8):
        sh = sharding.balanced_shards(rp, world)
        assert sh[0].row_lo == 0 and sh[-1].row_hi == 1000
        assert all(a.row_hi == b.row_lo for a, b in zip(sh, sh[1:]))
        assert sum(s.n_edges for s in sh) == rp[-1]
        assert max(s.n_edges for s in sh) - rp[-1] / world <= counts.max()


def test_balanced_shards_edge_cases():
    sh = sharding.balanced_shards([0], 4)  # no rows
    assert [s.n_rows for s in sh] == [0, 0, 0, 0]
    sh = sharding.balanced_shards([0, 0, 0], 2)  # rows without connections
    assert sum(s.n_rows for s in sh) == 2
    sh = sharding.balanced_shards([0, 100], 3)  # one heavy row
    assert sum(s.n_rows for s in sh) == 1 and sum(s.n_edges for s in sh) == 100
    with pytest.raises(ValueError):
        sharding.balanced_shards([0, 5, 3], 2)
    with pytest.raises(ValueError):
        sharding.even_shards(10, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        n_src, n_dst, n_edges = 300, 200, 5000
        L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=3)
        rp = np.searchsorted(L.to_id - n_src, np.arange(n_dst + 1)).astype(np.int64)
        shards = sharding.balanced_shards(rp, world)
        s = shards[rank]
        f = L.from_id[s.edge_lo:s.edge_hi].copy()
        t = (L.to_id[s.edge_lo:s.edge_hi] - np.uint32(s.row_lo)).copy()
        act = np.concatenate([L.act_in, np.zeros(s.n_rows, np.float32)])
        w, e, a = orc.step_hebbian(f, t, L.weight[s.edge_lo:s.edge_hi],
                                   L.trace[s.edge_lo:s.edge_hi], act, n_src, 0.9, 1e-3,
                                   sweeps=2)
        full = sharding.allgather_rows(torch.from_numpy(a[n_src:].copy()), shards)
        ws = [torch.zeros(n_edges, dtype=torch.float32) for _ in range(world)]
        wpad = torch.zeros(n_edges, dtype=torch.float32)
        wpad[s.edge_lo:s.edge_hi] = torch.from_numpy(w)
        dist.all_gather(ws, wpad)
        if rank == 0:
            q.put((full.numpy(), sum(x.numpy() for x in ws)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_one_process():
    from oracle import oracle as orc
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got_act, got_w = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_src, n_dst, n_edges = 300, 200, 5000
    L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=3)
    act = np.concatenate([L.act_in, np.zeros(n_dst, np.float32)])
    w, _, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, n_src, 0.9, 1e-3,
                               sweeps=2)
    np.testing.assert_array_equal(got_act.view(np.uint32), a[n_src:].view(np.uint32))
    np.testing.assert_array_equal(got_w.view(np.uint32), w.view(np.uint32))


def _owned_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L, size = 5, 12
        m = size // world
        t = torch.full((L * size,), -1.0)
        for l in range(L):  # each rank knows only its own units
            for u in range(rank * m, (rank + 1) * m):
                t[l * size + u] = 100 * l + u
        send = torch.empty(L * m)
        recv = torch.empty(world * L * m)
        sharding.allgather_owned(t, L, size, rank, world, send, recv)
        q.put((rank, t.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_allgather_owned_slices_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_owned_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.array([100 * l + u for l in range(5) for u in range(12)], np.float32)
    for r in range(world):
        np.testing.assert_array_equal(got[r], want)
