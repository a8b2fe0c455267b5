#!/usr/bin/env python
"""Benchmark: single sparse layer sweep (forward sum + fused per-connection
Hebbian trace update) -- connection updates per second and the fraction of
the HBM roofline.

Workload (per GPU): 2^20 source units, 2^20 destination units, 2^26 uniform
random (src, dst) connections stable-sorted by dst; weights N(0, 0.05^2),
inputs U(0, 1), traces 0; rule trace' = 0.9*trace + pre*post,
w' = w + 1e-3*trace'. One step = one sweep over all connections.
With --gpus N (one process per GPU, torchrun) the layer grows N-fold (weak
scaling): rank r owns destination rows [r*2^20, (r+1)*2^20) and a replica of
the N*2^20 source activations; after every sweep the destination slices are
all-gathered (NCCL over NVLink) as the hand-off to the next layer.

--impl reference times the reference implementation (its own headers
compiled from source, oracle/_ref) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("connection updates/sec (fwd+plasticity sweep) and % of HBM roofline "
          "at 1/2/4/8 B200")
UNIT = "connection-updates/s"
WORKLOAD = "single sparse layer sweep, fwd + fused Hebbian trace update"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n-src", type=int, default=1 << 20)
    p.add_argument("--n-dst", type=int, default=1 << 20)
    p.add_argument("--n-edges", type=int, default=1 << 26)
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="budget of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------------------
def measured_peak_gbs():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch(workload_key: str):
    f = ROOT / "profiles" / "traffic.json"
    if f.exists():
        d = json.loads(f.read_text())
        if workload_key in d:
            return d[workload_key]
    return None


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(prefix="plx_clocks_", suffix=".csv")
        self.proc = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------------------
def cpu_reference_sample(n_src, n_dst, n_edges, seed, budget_s, warmup=1, steps=None):
    """Times the reference implementation (oracle/_ref, all host threads, one
    reference network per destination-row shard) on a sample of the workload:
    the first 1/8 of the destination rows with their connections. Falls back
    to the oracle restatement (1 thread) when the reference build is absent."""
    import numpy as np

    from oracle import oracle
    from plastix_b200 import workloads

    frac = 8
    s_dst = max(1, n_dst // frac)
    s_edges = max(1, n_edges // frac)
    L = workloads.sparse_layer(n_src, s_dst, s_edges, seed=seed)
    threads = os.cpu_count() or 1
    R = oracle.ref()
    if R is not None:
        h = R.ref_sweep_shards_create(n_src, s_dst, s_edges, oracle._p(L.from_id),
                                      oracle._p(L.to_id), oracle._p(L.weight), threads,
                                      0.9, 1e-3)
        step = lambda: R.ref_sweep_shards_step(h, oracle._p(L.act_in))  # noqa: E731
        kind, cores = "reference", threads
    else:
        act = np.concatenate([L.act_in, np.zeros(s_dst, np.float32)])
        w, e = L.weight.copy(), L.trace.copy()
        acc = np.zeros(act.size, np.float32)

        def step():
            oracle.orc().oracle_step_hebbian(s_edges, oracle._p(L.from_id),
                                             oracle._p(L.to_id), None, oracle._p(w),
                                             oracle._p(e), oracle._p(act), act.size, n_src,
                                             0.9, 1e-3, oracle._p(acc))
        kind, cores = "port", 1
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if steps is not None:
            if n >= steps:
                break
        elif el >= budget_s and n >= 2:
            break
    el = time.perf_counter() - t0
    if R is not None:
        R.ref_sweep_shards_destroy(h)
    return {"value": s_edges * n / el, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": (f"{s_edges} connections into the first {s_dst} of {n_dst} "
                       f"destination rows (1/{frac} of the layer), {n} sweeps, "
                       f"{el:.2f} s"),
            "seconds_per_sweep": el / n}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cb = cpu_reference_sample(args.n_src, args.n_dst, args.n_edges, args.seed,
                              args.cpu_seconds, warmup=args.warmup, steps=args.steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cb["seconds_per_sweep"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "n_src": args.n_src, "n_dst": args.n_dst,
                   "n_edges": args.n_edges, "sample": cb["sample"]},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    from plastix_b200 import workloads
    from plastix_b200.runtime import Context, HebbianSweepLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)

    n_src_total = args.n_src * world
    n_dst = args.n_dst
    n_edges = args.n_edges
    ctx = Context(local)
    stream = ctx.stream

    # This rank's shard: rows [rank*n_dst, (rank+1)*n_dst) of the global layer,
    # sources over all n_src_total inputs.
    from_id, to_id, w, act_local = workloads.sparse_layer_device(
        n_src_total, n_dst, n_edges, args.seed + 7919 * rank, device)
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    act_src = torch.rand(n_src_total, generator=g, device=device)  # replicated inputs
    del act_local
    layer = HebbianSweepLayer(ctx, n_src_total, n_dst, from_id, to_id, w)
    del from_id, to_id, w
    gathered = torch.empty(n_dst * world, device=device) if world > 1 else None

    def step():
        out = layer.step(act_src)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)
        return out

    def barrier_sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timing -------------------------------------------
    for _ in range(args.warmup):
        step()
    barrier_sync()
    sampler = ClockSampler(local) if rank == 0 else None
    k0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        k0[i].record(stream)
        layer.step(act_src)
        k1[i].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered, layer.act_dst)
    t1.record(stream)
    barrier_sync()
    clocks = sampler.stop() if sampler else None
    ms = t0.elapsed_time(t1)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(k0, k1))
    if world > 1:
        t = torch.tensor([ms, kern_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kern_ms = float(t[0]), float(t[1])
    ms_per_step = ms / args.steps
    value = world * n_edges * args.steps / (ms / 1e3)

    # ---- end to end through the public API with host buffers --------------
    h_in = torch.rand(n_src_total, generator=torch.Generator().manual_seed(args.seed)
                      ).pin_memory()
    h_out = torch.empty(n_dst, pin_memory=True)
    dev_in = torch.empty(n_src_total, device=device)

    def e2e_step():
        dev_in.copy_(h_in, non_blocking=True)
        out = layer.step(dev_in)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)
        h_out.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier_sync()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier_sync()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t[0])
    e2e_value = world * n_edges * args.steps / (ems / 1e3)
    ctx.sync()

    # ---- roofline of the fused sweep kernel --------------------------------
    algo_bytes = 20 * n_edges + 8 * n_dst + 4 * n_src_total
    achieved = algo_bytes / (kern_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_reference_sample(args.n_src, args.n_dst, args.n_edges, args.seed,
                                  args.cpu_seconds)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded torch generator on device)",
        "config": {"workload": WORKLOAD, "n_src": n_src_total, "n_dst_per_gpu": n_dst,
                   "n_edges_per_gpu": n_edges, "parallelism": f"dst-range shards x{world}",
                   "l2": "inputs larger than L2: 1.36 GB of connection state streamed "
                         "per sweep vs 126 MB L2",
                   "handoff": "NCCL all-gather of destination activations per sweep"
                              if world > 1 else "none"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS hbm_gbs)",
                     "traffic": traffic_per_launch("sweep_hebbian_64M"),
                     "kernel_ms": kern_ms, "algorithmic_bytes_per_launch": algo_bytes},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": 4 * n_src_total * world,
                "d2h_bytes_per_step": 4 * n_dst * world},
        "clocks": clocks,
        "gpu_launches": args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
