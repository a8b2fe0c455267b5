"""Worker for tests/test_multigpu.py (one process per GPU, launched with
torch.distributed.run, any number of ranks up to 8): the sharded multilayer
iPC network against the same network on one GPU, the fused sweep + peer
hand-off against an NCCL all-gather, and a recurrent chain of hand-offs
against one GPU, all bit for bit. Not collected by pytest."""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from plastix_b200 import workloads  # noqa: E402
from plastix_b200.runtime import Context, HebbianSweepLayer, PredictiveCodingNet  # noqa: E402
from plastix_b200.sharding import PeerGather, ShardedPCNet, ipc_block_edges  # noqa: E402


def check_peer_handoff(ctx, rank, world, dev, layout):
    """The fused sweep + peer-memory hand-off against the plain sweep and an
    NCCL all-gather, over several steps (epochs)."""
    n_src, n_dst, n = 50_000, 40_000, 2_000_000
    f, t, w, _ = workloads.sparse_layer_device(n_src, n_dst, n, 100 + rank, dev)
    act = torch.rand(n_src, generator=torch.Generator(device=dev).manual_seed(9), device=dev)
    a = HebbianSweepLayer(ctx, n_src, n_dst, f, t, w.clone(), layout=layout)
    b = HebbianSweepLayer(ctx, n_src, n_dst, f, t, w.clone(), layout=layout)
    peer = PeerGather(ctx, n_dst * world, rank, world)
    want = torch.empty(n_dst * world, device=dev)
    got = torch.empty(n_dst * world, device=dev)
    bad = []
    for step in range(4):
        a.step_gather(act, peer, rank * n_dst)
        peer.barrier()
        dist.all_gather_into_tensor(want, b.step(act))
        peer.copy_to(got)
        ctx.sync()
        if not torch.equal(got, want):
            bad.append(f"peer hand-off ({layout}) step {step}")
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    dist.barrier()
    return bad


def check_peer_chain(ctx, rank, world, dev, layout, steps=6):
    """A recurrent layer whose sources are the previous step's gathered
    destination values, sharded by destination rows: each step's sweep reads
    the last epoch's hand-off buffer while faster ranks may already store the
    next epoch into the other buffer. Steps run back to back with no host
    synchronisation; the final activations and weights must equal the same
    layer stepped unsharded on one GPU, bit for bit."""
    m, per_rank = 16384, 1_000_000
    n = m * world  # sources = all ranks' destinations
    shards = [workloads.sparse_layer_device(n, m, per_rank, 300 + q, dev) for q in range(world)]
    act0 = torch.rand(n, generator=torch.Generator(device=dev).manual_seed(77), device=dev)
    f, t, w, _ = shards[rank]
    mine = HebbianSweepLayer(ctx, n, m, f, t, w.clone(), layout=layout)
    peer = PeerGather(ctx, n, rank, world)
    x = act0
    for _ in range(steps):
        mine.step_gather(x, peer, rank * m)
        peer.barrier()
        x = peer.gathered()
    # the same layer on one GPU: rank q's rows are rows [q*m, (q+1)*m)
    full = HebbianSweepLayer(
        ctx, n, n, torch.cat([s[0] for s in shards]),
        torch.cat([s[1] + q * m for q, s in enumerate(shards)]),
        torch.cat([s[2] for s in shards]).clone())
    y = act0
    for _ in range(steps):
        y = full.step(y).clone()
    ctx.sync()
    bad = []
    if not torch.equal(x, y):
        bad.append(f"peer chain ({layout}): gathered activations")
    lo = rank * per_rank
    if not torch.equal(mine.weight, full.weight[lo:lo + per_rank]):
        bad.append(f"peer chain ({layout}): weights")
    if not torch.equal(mine.trace, full.trace[lo:lo + per_rank]):
        bad.append(f"peer chain ({layout}): traces")
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    dist.barrier()
    return bad


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    S, F, L, seed, iters = 8192, 256, 5, 21, 3
    ctx = Context(local)
    net = ShardedPCNet(ctx, S, F, L, rank, world, seed)
    g = torch.Generator(device=dev).manual_seed(5)
    x0 = torch.rand(L * S, generator=g, device=dev) * 2 - 1
    inp = torch.rand(S, generator=g, device=dev)
    tgt = torch.rand(S, generator=g, device=dev) * 2 - 1
    net.x.copy_(x0)
    net.clamp(inp, tgt)
    for _ in range(iters):
        net.iteration()
    net.update()
    ref = PredictiveCodingNet(ctx, [S] * L,
                              [ipc_block_edges(l, S, F, seed, dev) for l in range(L - 1)],
                              layout="chunked")
    ref.x.copy_(x0)
    ref.clamp(inp, tgt)
    for _ in range(iters):
        ref.iteration()
    ref.update()
    ctx.sync()
    bad = []
    for l in range(1, L):
        if not torch.equal(net.own(net.err, l), net.own(ref.err, l)):
            bad.append(f"err layer {l}")
    for l in range(1, L - 1):
        if not torch.equal(net.own(net.x, l), net.own(ref.x, l)):
            bad.append(f"x layer {l}")
    for l in range(L - 1):
        a, b = net.lo * F, (net.lo + net.m) * F
        mine = net.fwd[l].weights_in_original_order(net.m * F)
        if not torch.equal(mine, ref.weights(l, S * F)[a:b]):
            bad.append(f"weights block {l}")
        if l in net.bwd:
            ch = net.bwd[l]
            valid = ch.perm >= 0
            full = ref.weights(l, S * F)
            if not torch.equal(ch.weight[valid], full[ch.perm[valid].long()]):
                bad.append(f"source-major weights block {l}")
    for layout in ("csr", "sliced"):
        bad += check_peer_handoff(ctx, rank, world, dev, layout)
        bad += check_peer_chain(ctx, rank, world, dev, layout)
    flag = torch.tensor([len(bad)], device=dev)
    dist.all_reduce(flag)
    if bad:
        print(f"rank {rank}: mismatch in {bad}", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(1 if int(flag.item()) else 0)


if __name__ == "__main__":
    main()
