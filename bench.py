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
import ctypes
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
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n-src", type=int, default=1 << 20)
    p.add_argument("--n-dst", type=int, default=1 << 20)
    p.add_argument("--n-edges", type=int, default=1 << 26)
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="budget of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-secondary", action="store_true",
                   help="N = 1: skip the other workloads' summaries in the headline line")
    p.add_argument("--handoff", choices=["p2p", "nccl"], default="p2p",
                   help="N > 1: hand the destination slices to every GPU with the sweep's "
                        "own stores over NVLink (p2p) or with an NCCL all-gather after it")
    p.add_argument("--layout", choices=["sliced", "csr"], default="sliced",
                   help="storage order of the swept layer: warp-sliced rows (one lane per "
                        "row) or the destination-sorted CSR order")
    p.add_argument("--api-traits", choices=["fused", "generic"], default="fused",
                   help="api workload: the rule as the library's HebbianTraceUpdate policy "
                        "(DoStep runs one fused sliced sweep) or as a user hook (the generic "
                        "device passes)")
    p.add_argument("--ipc-units", type=int, default=1 << 18,
                   help="units per layer of the ipc workload (2^18 in the configuration)")
    p.add_argument("--ipc-fan-in", type=int, default=2048)
    p.add_argument("--workload",
                   choices=["sweep", "swifttd", "ipc", "structural", "ceiling", "levels", "api",
                            "xor"],
                   default="sweep",
                   help="sweep: the single-layer fwd+Hebbian sweep (default, the headline); "
                        "swifttd: 4M-feature SwiftTD learner; ipc: 5-layer predictive-coding "
                        "net; structural: prune/regrow/re-sort/forward step; ceiling: the sweep "
                        "beside the same traffic without row folds and random gathers alone; "
                        "levels: RecomputeLevels + SortConnectionsByLevel at 2^24 connections; "
                        "api: the sweep through plastix::Network<Traits>::DoStep; "
                        "xor: the XOR MLP training run (launch-bound, DoSteps/s)")
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
            v = d[workload_key]
            return v["bytes_per_launch"] if isinstance(v, dict) else v
    return None


class ClockSampler:
    """Samples the SM clock and the clock-event reasons of one GPU while the
    timed region runs: NVML (read-only queries) from a thread every 2 ms, so
    even a timed region of a few milliseconds gets samples. Returns None when
    NVML is unavailable. Nothing is changed on the GPU."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4),
               ("hw_power_brake_slowdown", 0x80))

    def __init__(self, device_index: int):
        import threading

        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((float(mhz), int(rs)))
                    except Exception:
                        pass
                    self._stop.wait(0.002)

            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None

    def stop(self):
        if self._thread is None:
            return None
        self._stop.set()
        self._thread.join(timeout=2)
        if not self.samples:
            return None
        reasons = sorted({name for _, bits in self.samples for name, m in self.REASONS
                          if bits & m})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


def merge_clocks(per_rank):
    """One clock record for several GPUs: the lowest median SM clock, every
    reason any GPU reported, the sample counts added."""
    got = [c for c in per_rank if c]
    if not got:
        return None
    return {"sm_mhz": min(c["sm_mhz"] for c in got),
            "sm_max_mhz": max(c["sm_max_mhz"] or 0 for c in got),
            "reasons": sorted({r for c in got for r in c["reasons"]}),
            "samples": sum(c["samples"] for c in got), "gpus": len(got),
            "source": "nvml, every rank"}


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
    layer = HebbianSweepLayer(ctx, n_src_total, n_dst, from_id, to_id, w, layout=args.layout)
    del from_id, to_id, w
    gathered = torch.empty(n_dst * world, device=device) if world > 1 else None
    p2p = world > 1 and args.handoff == "p2p"
    peer = None
    if p2p:
        from plastix_b200.sharding import PeerGather
        peer = PeerGather(ctx, n_dst * world, rank, world)

    def sweep(x):
        """One sweep plus the hand-off of its destination slice to every GPU."""
        if p2p:
            out = layer.step_gather(x, peer, rank * n_dst)
            peer.barrier()
        else:
            out = layer.step(x)
            if world > 1:
                dist.all_gather_into_tensor(gathered, out)
        return out

    def step():
        return sweep(act_src)

    def barrier_sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def align_ranks():
        """Host barrier, then a device-side rendezvous on the timed stream, so
        every rank's first timed kernel starts together (a rank that arrives
        late cannot push its start-up delay into the others' timed region)."""
        barrier_sync()
        if p2p:
            peer.barrier()
        elif world > 1:
            dist.all_reduce(torch.zeros(1, device=device))

    # ---- device-resident timing -------------------------------------------
    for _ in range(args.warmup):
        step()
    sampler = ClockSampler(local)  # every rank samples its own GPU
    align_ranks()
    k0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k2 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        k0[i].record(stream)
        if p2p:
            layer.step_gather(act_src, peer, rank * n_dst)
        else:
            layer.step(act_src)
        k1[i].record(stream)
        if p2p:
            peer.barrier()
        elif world > 1:
            dist.all_gather_into_tensor(gathered, layer.act_dst)
        k2[i].record(stream)
    t1.record(stream)
    barrier_sync()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(k0, k1))
    handoff_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(k1, k2))
    if world > 1:
        t = torch.tensor([ms, kern_ms, handoff_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kern_ms, handoff_ms = float(t[0]), float(t[1]), float(t[2])
        every = [None] * world
        dist.all_gather_object(every, clocks)
        clocks = merge_clocks(every)
    ms_per_step = ms / args.steps
    value = world * n_edges * args.steps / (ms / 1e3)

    # ---- end to end through the public API with host buffers --------------
    # Every step copies its inputs from pinned host memory and reads its
    # destination activations back; the copies run on their own streams,
    # double-buffered, so step i+1's upload and step i's read-back overlap
    # the sweeps (the device-side hand-off of each step is unchanged). With
    # several GPUs each rank uploads only its own slice of the source vector
    # and the slices are all-gathered on the devices (NCCL over NVLink).
    n_in = n_src_total // world
    gen = torch.Generator().manual_seed(args.seed + rank)
    h_in = [torch.rand(n_in, generator=gen).pin_memory() for _ in range(2)]
    h_out = [torch.empty(n_dst, pin_memory=True) for _ in range(2)]
    dev_in = [torch.empty(n_src_total, device=device) for _ in range(2)]
    dev_out = [torch.empty(n_dst, device=device) for _ in range(2)]
    up = torch.cuda.Stream(device)
    down = torch.cuda.Stream(device)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, in_free = [ev(), ev()], [ev(), ev()]
    out_ready, out_free = [ev(), ev()], [ev(), ev()]
    for b in range(2):  # all buffers start free
        in_free[b].record(stream)
        out_free[b].record(stream)

    def e2e_step(i):
        b = i & 1
        up.wait_event(in_free[b])
        with torch.cuda.stream(up):
            if world > 1:
                mine = dev_in[b][rank * n_in:(rank + 1) * n_in]
                mine.copy_(h_in[b], non_blocking=True)
                dist.all_gather_into_tensor(dev_in[b], mine)
            else:
                dev_in[b].copy_(h_in[b], non_blocking=True)
        in_ready[b].record(up)
        stream.wait_event(in_ready[b])
        out = sweep(dev_in[b])
        in_free[b].record(stream)
        stream.wait_event(out_free[b])
        dev_out[b].copy_(out, non_blocking=True)
        out_ready[b].record(stream)
        down.wait_event(out_ready[b])
        with torch.cuda.stream(down):
            h_out[b].copy_(dev_out[b], non_blocking=True)
        out_free[b].record(down)

    for i in range(args.warmup):
        e2e_step(i)
    align_ranks()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    h0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_event(out_free[(args.steps - 1) & 1])  # the last read-back is inside
    e1.record(stream)
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # enqueue cost per step
    barrier_sync()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t[0])
        t = torch.tensor([host_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        host_ms = float(t[0])
    e2e_value = world * n_edges * args.steps / (ems / 1e3)
    ctx.sync()

    # ---- roofline of the fused sweep kernel --------------------------------
    algo_bytes = 20 * n_edges + 8 * n_dst + 4 * n_src_total
    achieved = algo_bytes / (kern_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()

    if world > 1:
        dist.barrier()
        if peer is not None:
            torch.cuda.synchronize()
            peer.close()
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
                   "layout": args.layout,
                   "l2": "inputs larger than L2: 1.36 GB of connection state streamed "
                         "per sweep vs 126 MB L2",
                   "handoff": ("destination slices stored by the sweep kernel into every "
                               "GPU's buffer over NVLink (peer memory), bounded barrier"
                               if p2p else "NCCL all-gather of destination activations per "
                               "sweep") if world > 1 else "none"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS hbm_gbs)",
                     "traffic": traffic_per_launch("sweep_hebbian_64M" if args.layout == "csr"
                                                   else "sweep_hebbian_sliced_64M"),
                     "kernel": "k_sweep_wtile" if args.layout == "csr" else "k_sweep_sliced",
                     "kernel_ms": kern_ms, "algorithmic_bytes_per_launch": algo_bytes},
        "handoff_ms": handoff_ms if world > 1 else None,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": 4 * n_in * world,
                "d2h_bytes_per_step": 4 * n_dst * world,
                "ms_per_step": ems / args.steps, "host_enqueue_ms_per_step": host_ms},
        "clocks": clocks,
        "gpu_launches": args.steps * (2 if p2p else 1),
    }
    if world == 1 and not args.no_secondary:
        ctx.sync()
        line["secondary"] = run_secondary()
    print(json.dumps(line), flush=True)
    return 0


# The other workloads, each run once in its own process after the headline
# measurement (one GPU): their own lines, summarised into the headline's
# "secondary" field, so that one default run records every configuration.
SECONDARY = ("swifttd", "structural", "levels", "ipc", "api", "xor")


def run_secondary() -> dict:
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    out = {}
    for name in SECONDARY:
        cmd = [sys.executable, str(ROOT / "bench.py"), "--workload", name, "--no-cpu-baseline",
               "--warmup", "3"]
        t0 = time.perf_counter()
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
            lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
            if r.returncode != 0 or not lines:
                out[name] = {"error": (r.stderr or r.stdout)[-300:]}
                continue
            d = json.loads(lines[-1])
            roof = d.get("roofline") or {}
            e2e = d.get("e2e") or {}
            clk = d.get("clocks") or {}
            out[name] = {"metric": d.get("metric"), "value": d.get("value"), "unit": d.get("unit"),
                         "ms_per_step": d.get("ms_per_step"),
                         "roofline_frac": roof.get("frac"), "e2e": e2e.get("value"),
                         "workload": (d.get("config") or {}).get("workload"),
                         "sm_mhz": clk.get("sm_mhz"), "clock_reasons": clk.get("reasons"),
                         "wall_s": round(time.perf_counter() - t0, 1)}
        except Exception as exc:  # one failing workload must not lose the headline
            out[name] = {"error": str(exc)[-300:]}
    return out


# ---------------------------------------------------------------------------
# The other configurations (single GPU): SwiftTD, iPC, structural plasticity.
# Each prints one JSON line of the same shape as the headline.
# ---------------------------------------------------------------------------
def _events(n):
    import torch
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def _timed_loop(stream, fn, steps, warmup, sampler_device=0):
    """W untimed calls, then K timed ones bracketed by synchronize; returns
    (total ms, clocks)."""
    import torch
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(sampler_device)
    t0, t1 = _events(2)
    t0.record(stream)
    for i in range(steps):
        fn(warmup + i)
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1), sampler.stop()


def _cpu_time(step, budget_s, min_steps=2):
    step()
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 >= budget_s and n >= min_steps:
            break
    return (time.perf_counter() - t0) / n


def _line(args, workload, value, unit, ms_per_step, config, roofline, cpu, e2e, clocks,
          launches, dtype="f32", extra=None):
    line = {"metric": METRIC if workload == "sweep" else f"{unit} ({workload})",
            "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded generators)", "config": config,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": launches}
    if args.impl == "reference":
        line = {"impl": "reference", "metric": line["metric"], "value": cpu["value"],
                "unit": cpu["unit"], "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "dtype": dtype,
                "data": line["data"], "config": config, "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": cpu["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if extra:
        line.update(extra)
    print(json.dumps(line), flush=True)


def _roof(bytes_per_launch, launch_ms, traffic_key):
    peak, kind = measured_peak_gbs()
    achieved = bytes_per_launch / (launch_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": f"{kind} (MEASURED_PEAKS hbm_gbs)",
            "traffic": traffic_per_launch(traffic_key), "kernel_ms": launch_ms,
            "algorithmic_bytes_per_launch": bytes_per_launch}


def bench_swifttd(args):
    """C4: 4,194,304 binary features, 20,971 active per step (seeded random
    sets), gamma 0.99, lambda 0.9, meta step size 1e-3, rewards N(0,1)."""
    import numpy as np
    import torch

    from plastix_b200.runtime import Context, SwiftTDLearner

    n, k, n_sets = 1 << 22, 20_971, 64
    torch.cuda.set_device(0)
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    sets = [torch.sort(torch.randperm(n, generator=g, device="cuda")[:k])[0].to(torch.int32)
            for _ in range(n_sets)]
    n_rw = max(args.steps + args.warmup, 64)
    rewards = torch.randn(n_rw, generator=g, device="cuda")
    td = SwiftTDLearner(ctx, n, gamma=0.99, lambda_=0.9, meta=1e-3, max_active=k)
    cpu = None
    if args.impl == "reference" or not args.no_cpu_baseline:
        cpu = _swifttd_cpu(args, n, k)
        if args.impl == "reference":
            return _line(args, "swifttd", None, "feature-updates/s", None,
                         {"workload": "SwiftTD", "n_features": n, "active": k}, None, cpu,
                         None, None, 0)
    ms, clocks = _timed_loop(ctx.stream, lambda i: td.step(sets[i % n_sets], rewards[i:i + 1]),
                             args.steps, args.warmup)
    # the dense pass alone (events between the two halves of the step)
    e = _events(2 * 20)
    for i in range(20):
        td.step_parts(sets[i % n_sets], rewards[i % n_rw:i % n_rw + 1],
                      between=lambda j=i: e[2 * j].record())
        e[2 * i + 1].record()
    torch.cuda.synchronize()
    dense_ms = statistics.mean(e[2 * i].elapsed_time(e[2 * i + 1]) for i in range(20))
    # end to end: each step's active list and reward from pinned host memory,
    # V back; uploads and read-backs on their own streams, double-buffered.
    h_sets = [s.cpu().pin_memory() for s in sets[:8]]
    h_rw = [rewards[i:i + 1].cpu().pin_memory() for i in range(8)]
    d_idx = [torch.empty(k, dtype=torch.int32, device="cuda") for _ in range(2)]
    d_rw = [torch.empty(1, device="cuda") for _ in range(2)]
    h_v = [torch.empty(1, pin_memory=True) for _ in range(2)]
    d_v = [torch.empty(1, device="cuda") for _ in range(2)]
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    for b in range(2):
        in_free[b].record(ctx.stream)
        out_free[b].record(ctx.stream)

    def e2e(i):
        b = i & 1
        up.wait_event(in_free[b])
        with torch.cuda.stream(up):
            d_idx[b].copy_(h_sets[i % 8], non_blocking=True)
            d_rw[b].copy_(h_rw[i % 8], non_blocking=True)
        in_ready[b].record(up)
        ctx.stream.wait_event(in_ready[b])
        v = td.step(d_idx[b], d_rw[b])
        in_free[b].record(ctx.stream)
        ctx.stream.wait_event(out_free[b])
        d_v[b].copy_(v, non_blocking=True)
        out_ready[b].record(ctx.stream)
        down.wait_event(out_ready[b])
        with torch.cuda.stream(down):
            h_v[b].copy_(d_v[b], non_blocking=True)
        out_free[b].record(down)

    def e2e_timed():
        for i in range(args.warmup):
            e2e(i)
        torch.cuda.synchronize()
        t0, t1 = _events(2)
        t0.record(ctx.stream)
        up.wait_event(t0)
        for i in range(args.steps):
            e2e(i)
        ctx.stream.wait_event(out_free[(args.steps - 1) & 1])
        t1.record(ctx.stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)
    ems = e2e_timed()
    ctx.sync()
    value = n * args.steps / (ms / 1e3)
    algo = 72 * n  # dense pass: 8 fields read, 10 written, 4 B each
    _line(args, "swifttd", value, "feature-updates/s", ms / args.steps,
          {"workload": "SwiftTD linear TD learner", "n_features": n, "active_per_step": k,
           "gamma": 0.99, "lambda": 0.9, "meta": 1e-3,
           "l2": "inputs larger than L2: 168 MB of per-feature state per step"},
          _roof(algo, dense_ms, "swifttd_dense_4M"), cpu,
          {"value": n * args.steps / (ems / 1e3), "unit": "feature-updates/s",
           "h2d_bytes_per_step": 4 * k + 4, "d2h_bytes_per_step": 4},
          clocks, 3 * args.steps,
          extra={"dense_pass_ms": dense_ms, "step_overhead_ms": ms / args.steps - dense_ms})


def _swifttd_cpu(args, n, k):
    import numpy as np

    from oracle import oracle
    rng = np.random.default_rng(args.seed)
    f = np.zeros(n, np.float32)
    f[rng.choice(n, k, replace=False)] = 1.0
    R = oracle.ref()
    if R is not None:
        feats = f[None, :]
        rw = np.zeros(1, np.float32)
        out = np.empty((10, n), np.float32)
        v = np.empty(1, np.float32)

        def step():  # network construction excluded below: time DoStep only
            R.ref_swifttd_example_run(n, oracle._p(feats), oracle._p(rw), 1, 0.05,
                                      oracle._p(out), oracle._p(v))
        t_one = _cpu_time(step, args.cpu_seconds / 2, 1)
        feats3 = np.repeat(f[None, :], 3, axis=0)
        rw3 = np.zeros(3, np.float32)

        def step3():
            R.ref_swifttd_example_run(n, oracle._p(feats3), oracle._p(rw3), 3, 0.05,
                                      oracle._p(out), oracle._p(v))
        t_three = _cpu_time(step3, args.cpu_seconds / 2, 1)
        per_step = max((t_three - t_one) / 2, 1e-9)
        return {"value": n / per_step, "unit": "feature-updates/s", "cores": 1,
                "kind": "reference",
                "sample": f"reference SwiftTD example network ({n} features, {k} active; its "
                          "fixed gamma 1.0, same work per step), DoStep time from runs of 1 and 3 "
                          "steps (construction cancels out)"}
    fields = oracle.td_fields(n)
    g = oracle.td_globals()
    per_step = _cpu_time(lambda: oracle.swifttd_step(fields, f, 0.5, g), args.cpu_seconds, 2)
    return {"value": n / per_step, "unit": "feature-updates/s", "cores": 1, "kind": "port",
            "sample": f"oracle SwiftTD step, {n} features, {k} active"}


def bench_ipc(args):
    """C5: 5 layers of 262,144 units, 2,048 random sources per destination
    (2^31 connections), weights N(0, 1/2048), inputs U(0,1); a sample = 20
    inference iterations (forward, Pipeline backward, value update) + one
    weight update. One timed step = one sample. With --gpus N the same
    network is sharded by unit range over N GPUs (strong scaling; all-gathers
    of f(x) and eps per iteration)."""
    import torch
    import torch.distributed as dist

    from plastix_b200.runtime import Context
    from plastix_b200.sharding import ShardedPCNet

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    S, F, iters, L = args.ipc_units, args.ipc_fan_in, 20, 5
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    else:  # a one-rank group keeps the all-gathers on the same code path
        dist.init_process_group("nccl", init_method=f"file://{tempfile.mktemp(prefix='plx_pg_')}",
                                rank=0, world_size=1, device_id=dev)
    ctx = Context(local)
    net = ShardedPCNet(ctx, S, F, L, rank, world, args.seed, gamma=0.1, alpha=0.005)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    inputs = torch.rand(S, generator=g, device=dev)
    targets = torch.rand(S, generator=g, device=dev) * 2 - 1
    E, Eb = (L - 1) * S * F, (L - 2) * S * F

    def sample(i):
        net.clamp(inputs, targets)
        for _ in range(iters):
            net.iteration()
        net.update()
    steps = max(1, min(args.steps, 5))
    for _ in range(min(args.warmup, 3)):
        sample(0)
    dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    t0, t1 = _events(2)
    t0.record(ctx.stream)
    for i in range(steps):
        sample(i)
    t1.record(ctx.stream)
    dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    ms = t0.elapsed_time(t1)
    # the dominant sweep alone: the forward folds of this rank's rows
    e = _events(2)
    e[0].record(ctx.stream)
    for _ in range(5):
        for l, ch in enumerate(net.fwd):
            ch.fold(net.layer(net.act, l), net.own(net.err, l + 1), 3,
                    value=net.own(net.x, l + 1))
    e[1].record(ctx.stream)
    torch.cuda.synchronize()
    fwd_ms = e[0].elapsed_time(e[1]) / 5
    t = torch.tensor([ms, fwd_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms = float(t[0]), float(t[1])
    ctx.sync()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return 0
    visits = iters * (E + Eb) + (E + Eb)
    per_sample = ms / steps
    cpu = None if (world > 1 or args.no_cpu_baseline) else ipc_cpu_sample(F, iters, args.seed)
    line = {"metric": "connection-visits/s (ipc)", "value": visits / (per_sample / 1e3),
            "unit": "connection-visits/s", "n_gpus": world, "steps": steps,
            "warmup": min(args.warmup, 3), "ms_per_step": per_sample, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (counter-based hash generator)",
            "config": {"workload": "multilayer sparse predictive coding (iPC)", "layers": L,
                       "units_per_layer": S, "fan_in": F, "connections": E,
                       "iterations_per_sample": iters,
                       "parallelism": f"unit-range shards x{world}, NCCL all-gather of f(x) "
                                      "and eps per iteration",
                       "counting": "per sample: 20 x (forward over all connections + backward "
                                   "over the hidden-source ones) + one update of both copies",
                       "layout": "chunked-source (16-bit source offsets, 16384-source chunks "
                                 "in shared memory)",
                       "roofline_bytes": "forward: 6 B per connection (16-bit offset + weight)",
                       "l2": "inputs larger than L2"},
            "roofline": _roof(6 * E / world, fwd_ms, "ipc_forward_2G"),
            "cpu_baseline": cpu, "e2e": None, "clocks": clocks, "gpu_launches": None,
            "forward_ms": fwd_ms}
    print(json.dumps(line), flush=True)
    return 0


def ipc_cpu_sample(fan_in, iters, seed, units=4096, layers=5):
    """One iPC sample (clamp + pre-step, `iters` x (forward, backward, value
    update), one weight update) of the same network scaled to `units` per
    layer, through the oracle's C restatement on one host thread: the CPU
    baseline of the iPC workload (the full network does not fit a bounded
    CPU sample)."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(seed)
    begin = [l * units for l in range(layers + 1)]
    frm, to, w = [], [], []
    for l in range(layers - 1):
        to.append(np.repeat(np.arange(units, dtype=np.uint32) + np.uint32(begin[l + 1]), fan_in))
        frm.append((rng.integers(0, units, units * fan_in) + begin[l]).astype(np.uint32))
        w.append(rng.normal(0, 1 / np.sqrt(fan_in), units * fan_in).astype(np.float32))
    frm, to, w = np.concatenate(frm), np.concatenate(to), np.concatenate(w)
    n = begin[-1]
    hidden = (begin[1], begin[-2])
    x = rng.uniform(-1, 1, n).astype(np.float32)
    inputs = rng.uniform(0, 1, units).astype(np.float32)
    x[begin[-2]:] = rng.uniform(-1, 1, units).astype(np.float32)
    t0 = time.perf_counter()
    x[:units] = inputs
    act = orc.ipc_prestep(x, inputs, hidden)
    err = None
    for _ in range(iters):
        err = orc.ipc_forward(frm, to, w, act, x, units)
        bu = orc.ipc_backward(frm, to, w, err, x, hidden)
        orc.ipc_hidden_update(x, err, bu, act, 0.1, hidden)
    w = orc.update_post(frm, to, act, err, w, 2, 0.005)
    secs = time.perf_counter() - t0
    e, eb = frm.size, (layers - 2) * units * fan_in
    visits = iters * (e + eb) + e
    return {"value": visits / secs, "unit": "connection-visits/s", "cores": 1, "kind": "port",
            "sample": f"one sample of the network scaled to {units} units per layer "
                      f"({e} connections, fan-in {fan_in}): {secs:.2f} s, oracle C "
                      "restatement, one thread"}


def bench_structural(args):
    """C3: 2^23 sources, 2^23 destinations, 2^24 connections dst-sorted,
    w N(0, 0.1^2), u8 age; prune |w| < 0.02 by compaction, regrow the same
    number, re-sort by destination (the regrown tail radix-sorted and merged
    with the survivors), row offsets, forward sweep (one thread per row).
    Under torchrun each rank
    holds its own destination shard of that size (weak scaling): compaction,
    regrowth (rank-keyed seed) and the re-sort are shard-local, so no
    collective touches the step; the barrier and the max over ranks only
    bracket the timing."""
    import torch
    import torch.distributed as dist

    from plastix_b200.runtime import Context, StructuralLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    n_src = n_dst = 1 << 23
    n = 1 << 24
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    ctx = Context(local)
    g = torch.Generator(device=dev).manual_seed(args.seed + 7919 * rank)
    src = torch.randint(0, n_src, (n,), generator=g, device=dev)
    dst = torch.randint(0, n_dst, (n,), generator=g, device=dev)
    dst, order = torch.sort(dst, stable=True)
    f = src[order].to(torch.int32)
    t = (dst + n_src).to(torch.int32)
    w = torch.randn(n, generator=g, device=dev) * 0.1
    age = torch.randint(0, 256, (n,), generator=g, device=dev).to(torch.uint8)
    act = torch.rand(n_src, generator=g, device=dev)
    del src, dst, order
    layer = StructuralLayer(ctx, n_src, n_dst, f, t, w, age, threshold=0.02, seed=11 + rank)
    steps = max(1, min(args.steps, 50))
    for _ in range(args.warmup):
        layer.step(act)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    t0, t1 = _events(2)
    t0.record(ctx.stream)
    for _ in range(steps):
        layer.step(act)
    t1.record(ctx.stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    ms = t0.elapsed_time(t1)
    if world > 1:
        tm = torch.tensor([ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm[0])
        dist.barrier()
        dist.destroy_process_group()
    ctx.sync()
    if rank != 0:
        return 0
    cpu = None if (world > 1 or args.no_cpu_baseline) else structural_cpu_sample(
        n_src // 8, n_dst // 8, n // 8, args.seed)
    _line(args, "structural", world * n * steps / (ms / 1e3), "connections/s", ms / steps,
          {"workload": "structural plasticity step", "n_src": n_src, "n_dst_per_gpu": n_dst,
           "connections_per_gpu": n, "prune": "|w| < 0.02", "steps": steps,
           "parallelism": f"destination shards x{world}, shard-local (no collective)"},
          None, cpu, None, clocks, None, extra={"n_gpus": world})
    return 0


def structural_cpu_sample(n_src, n_dst, n, seed, steps=3):
    """The structural step (prune by compaction, regrowth, stable re-sort by
    destination, forward) through the oracle's C restatement on one host
    thread, on the workload scaled by 1/8: the CPU baseline."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(seed)
    t = np.sort(rng.integers(0, n_dst, n)).astype(np.uint32) + np.uint32(n_src)
    f = rng.integers(0, n_src, n).astype(np.uint32)
    w = (rng.standard_normal(n) * 0.1).astype(np.float32)
    age = rng.integers(0, 256, n).astype(np.uint8)
    act = np.concatenate([rng.random(n_src, dtype=np.float32), np.zeros(n_dst, np.float32)])
    t0 = time.perf_counter()
    for s in range(steps):
        f, t, w, age, _ = orc.structural_step(f, t, w, age, n_src, n_dst, 0.02, 11, s * n)
        orc.forward_pipeline(f, t, w, act, n_src)
    secs = time.perf_counter() - t0
    return {"value": n * steps / secs, "unit": "connections/s", "cores": 1, "kind": "port",
            "sample": f"{steps} steps on the workload scaled by 1/8 ({n} connections, "
                      f"{n_src} + {n_dst} units): {secs:.2f} s, oracle C restatement, "
                      "one thread"}


def _probe_lib():
    """The measurement-only library of the ceiling workload (its kernels are
    not part of the product library)."""
    from ctypes import POINTER, c_float, c_int, c_uint32, c_uint64, c_void_p

    from plastix_b200 import _abi, build

    _abi.lib()  # the product library first: the probes use its contexts
    lib = ctypes.CDLL(str(build.PROBE_LIB))
    lib.plx_probe_gather.restype = c_int
    lib.plx_probe_gather.argtypes = [c_void_p, c_void_p, c_uint32, c_uint64, c_void_p,
                                     POINTER(c_uint64)]
    lib.plx_probe_sweep_nofold.restype = c_int
    lib.plx_probe_sweep_nofold.argtypes = [c_void_p, c_uint64, c_void_p, c_void_p, c_uint32,
                                           c_void_p, c_void_p, c_float, c_float, c_void_p,
                                           c_void_p]
    return lib


def bench_ceiling(args):
    """The sweep (CSR order and warp-sliced rows) against the two pieces of its
    traffic no fold order removes: the same connections swept without the row
    folds (FromId/Weight/Trace loads, act[FromId] gathers, Weight/Trace
    stores) and as many random gathers alone; and the shared-memory
    source-chunk route. Prints per-launch times (CUDA events, inputs > L2)."""
    import torch

    from plastix_b200 import _abi, workloads
    from plastix_b200.runtime import Context, HebbianSweepLayer

    ctx = Context(0)
    probe = _probe_lib()
    device = ctx.device
    n_src, n_dst, n = args.n_src, args.n_dst, args.n_edges
    from_id, to_id, w, act = workloads.sparse_layer_device(n_src, n_dst, n, args.seed, device)
    layer = HebbianSweepLayer(ctx, n_src, n_dst, from_id, to_id, w.clone())
    e = torch.zeros(n, device=device)
    w2, e2 = torch.empty_like(w), torch.empty_like(e)
    sink = torch.zeros(1, device=device)
    done = ctypes.c_uint64(0)

    def probe_call(name, *a):
        rc = getattr(probe, name)(*a)
        if rc != 0:
            raise _abi.PlxError(rc, name, _abi.lib().plx_last_error().decode())

    def nofold(i):
        probe_call("plx_probe_sweep_nofold", ctx.handle, n, from_id.data_ptr(), act.data_ptr(),
                   n_src, w.data_ptr(), e.data_ptr(), 0.9, 1e-3, w2.data_ptr(), e2.data_ptr())

    def gather(i):
        probe_call("plx_probe_gather", ctx.handle, act.data_ptr(), n_src, n, sink.data_ptr(),
                   ctypes.byref(done))

    sliced = HebbianSweepLayer(ctx, n_src, n_dst, from_id, to_id, w.clone(), layout="sliced")
    out = {}
    for name, fn in (("sweep", lambda i: layer.step(act)), ("sliced", lambda i: sliced.step(act)),
                     ("nofold", nofold), ("gather", gather)):
        ms, clocks = _timed_loop(ctx.stream, fn, args.steps, args.warmup)
        out[name] = ms / args.steps
    ctx.sync()
    gathers = int(done.value)
    # The shared-memory source-chunk route for the same layer (the layout the
    # multilayer iPC uses): rows' connections grouped by 16384-source chunk,
    # chunk partials added per row, then an update pass. Timed with the
    # trace-free Hebbian update, so both times are lower bounds for the
    # fused rule.
    from plastix_b200.runtime import ChunkedRows
    del layer, sliced, e, w2, e2
    torch.cuda.empty_cache()
    ch = ChunkedRows(ctx, from_id, to_id, w, 0, n_src, n_src, n_dst)
    post = torch.empty(n_dst, device=device)
    ms_f, _ = _timed_loop(ctx.stream, lambda i: ch.fold(act, post, _abi.APPLY_IDENTITY),
                          args.steps, args.warmup)
    ms_u, _ = _timed_loop(ctx.stream, lambda i: ch.update(act, post, _abi.UPDATE_HEBBIAN, 1e-3),
                          args.steps, args.warmup)
    ctx.sync()
    out["chunked_fold"], out["chunked_update"] = ms_f / args.steps, ms_u / args.steps
    chunk_slots = int(ch.seg_ptr[-1].item())
    del ch
    line = {"metric": "ms per launch (sweep memory ceiling probes)", "unit": "ms",
            "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "dtype": "f32", "data": "synthetic (seeded generators)",
            "config": {"workload": "sweep ceiling probes", "n_src": n_src, "n_dst": n_dst,
                       "connections": n, "l2": "inputs larger than L2"},
            "sweep_ms": out["sweep"], "sliced_sweep_ms": out["sliced"],
            "nofold_ms": out["nofold"], "gather_ms": out["gather"],
            "gathers": gathers, "gathers_per_s": gathers / (out["gather"] / 1e3),
            "sweep_over_nofold": out["sweep"] / out["nofold"],
            "chunked_fold_ms": out["chunked_fold"], "chunked_update_ms": out["chunked_update"],
            "chunked_slots_per_connection": chunk_slots / n, "clocks": clocks}
    print(json.dumps(line), flush=True)
    ctx.close()


def bench_levels(args):
    """Level re-sort after a structural step, Topological model, at the
    structural configuration's size (2^23 input units, 2^23 destination
    units, 2^24 connections, FromId/ToId/Weight/Age fields): RecomputeLevels
    then SortConnectionsByLevel (SrcLevel refresh, stable radix sort on the
    16-bit key, Gather of every field). The unit is connections per second
    of the whole re-sort; the roofline is taken on RecomputeLevels alone."""
    import numpy as np
    import torch

    from plastix_b200.runtime import (Context, Scratch, recompute_levels,
                                      sort_connections_by_level)

    ctx = Context(0)
    device = ctx.device
    n_in, n = 1 << 23, 1 << 24
    n_units = 2 * n_in
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    f = torch.randint(0, n_in, (n,), generator=g, device=device, dtype=torch.int32)
    t = torch.randint(n_in, n_units, (n,), generator=g, device=device, dtype=torch.int32)
    w = torch.randn(n, generator=g, device=device)
    age = torch.randint(0, 256, (n,), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    level = torch.zeros(n_units, dtype=torch.int16, device=device)
    outs = [torch.empty_like(x) for x in (f, t, w, age)]
    pairs = list(zip((f, t, w, age), outs))
    scr = Scratch(device)

    def resort(i):
        sort_connections_by_level(ctx, n_units, n_in, f, t, level, pairs, scratch=scr)

    def recompute(i):
        recompute_levels(ctx, n_units, n_in, f, t, level, scratch=scr)

    ms_r, _ = _timed_loop(ctx.stream, recompute, args.steps, args.warmup)
    ms, clocks = _timed_loop(ctx.stream, resort, args.steps, args.warmup)
    ctx.sync()
    rec_ms, step_ms = ms_r / args.steps, ms / args.steps
    # minimum traffic of RecomputeLevels: FromId + ToId once, every level written
    roof = _roof(8 * n + 2 * n_units, rec_ms, "levels_recompute_16M")
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle
        fh = f.cpu().numpy().view(np.uint32)
        th = t.cpu().numpy().view(np.uint32)
        sec = _cpu_time(lambda: oracle.sort_connections_by_level(n_units, n_in, fh, th),
                        budget_s=8.0, min_steps=1)
        cpu = {"value": n / sec, "unit": "connections/s", "cores": 1, "kind": "port",
               "sample": "oracle restatement of RecomputeLevels + stable level sort, full "
                         "size, one thread (fields not gathered)"}
    _line(args, "levels", n / (step_ms / 1e3), "connections/s", step_ms,
          {"workload": "level re-sort (RecomputeLevels + SortConnectionsByLevel)",
           "n_units": n_units, "n_input": n_in, "connections": n,
           "fields": "FromId, ToId, Weight, Age", "recompute_ms": rec_ms},
          roof, cpu, None, clocks, None)
    ctx.close()


def bench_api(args):
    """The single-layer sweep through the reference's C++ API: a
    plastix::Network<Traits> with PLASTIX_HD Hebbian-trace policies
    (plastix_b200/apps/network_sweep.cu), stepped with DoStep; --api-traits
    picks the library policy (fused route) or the user-hook spelling. Device time
    per DoStep from CUDA events on the network's stream; e2e per step is
    DoStep from a host input vector + GetOutput (host clock)."""
    from plastix_b200 import build

    exe = build.app_path("network_sweep")
    if not exe.exists():
        exe = build.build_app("network_sweep")
    # clocks are sampled over the program's timed loops only (it announces
    # them on stdout), not over the host-side construction of the network;
    # the sampler is started first, so that its set-up does not eat into a
    # short timed region, and its samples are cleared at the announcement
    sampler = ClockSampler(0)
    proc = subprocess.Popen([str(exe), "bench", str(args.n_src), str(args.n_dst),
                             str(args.n_edges), str(args.seed), str(args.steps),
                             str(args.warmup), args.api_traits], stdout=subprocess.PIPE,
                            stderr=subprocess.PIPE, text=True)
    lines, began = [], False
    for line in proc.stdout:
        lines.append(line)
        if line.startswith("timed-region-begins"):
            sampler.samples.clear()
            began = True
    rc = proc.wait(timeout=1800)
    clocks = sampler.stop()
    if not began:
        clocks = None
    if rc != 0:
        raise SystemExit(f"network_sweep failed:\n{''.join(lines)}\n{proc.stderr.read()}")
    d = json.loads(lines[-1])
    n = args.n_edges
    ms = d["device_ms_per_step"]
    algo = 20 * n + 8 * args.n_dst + 4 * args.n_src
    route = ("HebbianTraceUpdate policy: one fused sliced sweep per DoStep"
             if args.api_traits == "fused" else
             "user hook: generic passes (tiled forward, per-connection update)")
    config = {"workload": "single sparse layer sweep through plastix::Network<Traits>::DoStep "
                          "(PLASTIX_HD policies: identity forward, Hebbian trace update)",
              "traits": route, "n_src": args.n_src, "n_dst": args.n_dst, "n_edges": n,
              "l2": "inputs larger than L2", "build_s": d["build_s"]}
    e2e = {"value": n / (d["e2e_ms_per_step"] / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": 4 * args.n_src, "d2h_bytes_per_step": 4 * args.n_dst}
    _line(args, "api", n / (ms / 1e3), UNIT, ms, config, _roof(algo, ms, None), None, e2e,
          clocks, None)
    return 0


def bench_xor(args):
    """The XOR MLP (2 -> 8 -> 1 sigmoid, MSE, backward, gradient step at 0.5;
    5,000 epochs of four DoSteps, each followed by GetOutput) through the
    device Network: plastix_b200/apps/xor_train.cu, with DoStep as one kernel
    of one CTA (the value), replayed as a CUDA graph and with every pass
    launched (both in the config).
    A 24-connection network is launch- and latency-bound: the number is
    DoSteps per second of wall time around the epoch loop, host inputs in and
    the output read back every step. The baseline is the same program built
    against the reference's headers (oracle/_ref/xor_train) on one core."""
    from plastix_b200 import build

    exe = build.app_path("xor_train")
    if not exe.exists():
        exe = build.build_app("xor_train")
    epochs = 5000

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        if r.returncode != 0:
            raise SystemExit(f"{cmd[0]} failed:\n{r.stdout}\n{r.stderr}")
        return json.loads(r.stdout.strip().splitlines()[-1])

    cpu = None
    ref = ROOT / "oracle" / "_ref" / "xor_train"
    if ref.exists() and not args.no_cpu_baseline:
        best = min(run([str(ref), str(epochs)])["train_s"] for _ in range(3))
        cpu = {"value": 4 * epochs / best, "unit": "steps/s", "cores": 1, "kind": "reference",
               "sample": f"the whole run: {epochs} epochs, {4 * epochs} DoSteps (best of 3)"}
    if args.impl == "reference":
        if cpu is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/xor_train "
                              "was not built (the reference tree was absent at build time)"}))
            return 0
        _line(args, "xor", cpu["value"], "steps/s", 1e3 / cpu["value"], {"workload": "xor"},
              None, cpu, None, None, None)
        return 0
    sampler = ClockSampler(0)
    g = run([str(exe), str(epochs), "single"])
    clocks = sampler.stop()
    r = run([str(exe), str(epochs), "graph"])
    e = run([str(exe), str(epochs), "eager"])
    steps = g["steps"]
    value = steps / g["train_s"]
    config = {"workload": "XOR MLP training through Network<Traits>::DoStep (2 -> 8 -> 1 "
                          "sigmoid, MSE, backward, gradient descent, Topological)",
              "epochs": epochs, "do_steps": steps, "step": "one kernel of one CTA per DoStep",
              "graph_replay_steps_per_s": r["steps"] / r["train_s"],
              "eager_steps_per_s": e["steps"] / e["train_s"], "final_loss": g["final_loss"],
              "final_losses_equal": g["final_loss"] == r["final_loss"] == e["final_loss"],
              "xor_solved": g["pass"] and r["pass"] and e["pass"]}
    e2e = {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4}
    _line(args, "xor", value, "steps/s", 1e3 * g["train_s"] / steps, config, None, cpu, e2e,
          clocks, None)
    return 0


def run_other(args):
    if args.gpus != 1 and args.workload not in ("ipc", "structural"):
        raise SystemExit(f"--workload {args.workload} runs on one GPU")
    return {"swifttd": bench_swifttd, "ipc": bench_ipc, "structural": bench_structural,
            "ceiling": bench_ceiling, "levels": bench_levels, "api": bench_api,
            "xor": bench_xor}[args.workload](
                args) or 0


def main():
    args = parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    if args.workload != "sweep":
        return run_other(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
