"""Regenerates the golden fixtures in this folder by running the REFERENCE
implementation (oracle/_ref, compiled from the reference sources by
oracle/build.py). Run from the repository root: python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build as ob  # noqa: E402
from oracle import oracle  # noqa: E402
from plastix_b200 import workloads  # noqa: E402

HERE = Path(__file__).resolve().parent


def sweep_hebbian_small():
    n_src, n_dst, n_edges, seed, sweeps, decay, rate = 256, 128, 4096, 7, 3, 0.9, 1e-3
    L = workloads.sparse_layer(n_src, n_dst, n_edges, seed=seed)
    w, e, a = oracle.ref_sweep_run(n_src, n_dst, L.from_id, L.to_id, L.weight, L.trace,
                                   L.act_in, sweeps, decay, rate)
    np.savez_compressed(HERE / "sweep_hebbian_small.npz", n_src=n_src, n_dst=n_dst,
                        n_edges=n_edges, seed=seed, sweeps=sweeps, decay=decay, rate=rate,
                        w=w, trace=e, act=a)


if __name__ == "__main__":
    ob.build()
    if oracle.ref() is None:
        sys.exit("reference build missing: the reference tree is needed to make fixtures")
    sweep_hebbian_small()
    print("fixtures written to", HERE)
