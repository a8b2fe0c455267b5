"""Regenerates the golden fixtures in this folder by running the REFERENCE
implementation (oracle/_ref, compiled from the reference sources by
oracle/build.py). Run from the repository root: python tests/golden/make_golden.py
[fixture names]
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


def swifttd_features(n, steps, seed):
    """Seeded feature rows for the SwiftTD fixtures: 0, 1, 2 or 5 active
    features per step (one active feature keeps Tau <= Eta, so both branches
    of swifttd.cpp:169-185 occur), value 1.0; rewards N(0, 1)."""
    rng = np.random.default_rng(seed)
    feats = np.zeros((steps, n), np.float32)
    for s in range(steps):
        # the last steps have one active feature, so the final H/ZBar are live
        k = 1 if s >= steps - 6 else rng.choice([0, 1, 1, 1, 2, 5])
        feats[s, rng.choice(n, k, replace=False)] = 1.0
    return feats, rng.normal(size=steps).astype(np.float32)


def swifttd_small():
    n, steps, seed = 64, 200, 5
    feats, rewards = swifttd_features(n, steps, seed)
    fields, v = oracle.ref_swifttd_example_run(feats, rewards, alpha_init=0.05)
    np.savez_compressed(HERE / "swifttd_small.npz", n=n, steps=steps, seed=seed,
                        features=feats, rewards=rewards, fields=fields, v=v)


XOR_INPUTS = np.array([[0, 0], [0, 1], [1, 0], [1, 1]], np.float32)
XOR_TARGETS = np.array([0, 1, 1, 0], np.float32)


def mlp_xor_small():
    """The XOR MLP (2 -> 8 -> 1, RandomUniformWeight seed 1234) trained by the
    reference with mlp_xor.cpp's policies: initial and final weights and the
    final predictions after 200 and after 5000 epochs."""
    w0, w200, p200 = oracle.ref_mlp_run(2, 8, 1234, 200, XOR_INPUTS, XOR_TARGETS)
    _, w5000, p5000 = oracle.ref_mlp_run(2, 8, 1234, 5000, XOR_INPUTS, XOR_TARGETS)
    np.savez_compressed(HERE / "mlp_xor_small.npz", inputs=XOR_INPUTS, targets=XOR_TARGETS,
                        seed=1234, w_init=w0, w_200=w200, preds_200=p200, w_5000=w5000,
                        preds_5000=p5000)


def ipc_small():
    """30 steps of the iPC example's own iPCStep (3 -> 16 -> 1) from seeded
    weights and value nodes."""
    rng = np.random.default_rng(3)
    n_conn, n_units, steps = 3 * 16 + 16, 20, 30
    w = rng.uniform(-0.5, 0.5, n_conn).astype(np.float32)
    x = rng.uniform(-1, 1, n_units).astype(np.float32)
    inputs = rng.uniform(-1, 1, (steps, 3)).astype(np.float32)
    targets = rng.normal(size=steps).astype(np.float32)
    rw, rx, rerr = oracle.ref_ipc_run(inputs, targets, w, x)
    np.savez_compressed(HERE / "ipc_small.npz", w0=w, x0=x, inputs=inputs, targets=targets,
                        w=rw, x=rx, err=rerr)


LEVEL_CASES = {  # name: (n_units, n_input, n_conns, seed, back_edges, dead_frac, into_inputs)
    "dag": (3000, 40, 12000, 1, 0, 0.0, 0),
    "cyclic": (3000, 40, 12000, 2, 30, 0.0, 0),
    "dead": (3000, 40, 12000, 3, 0, 0.15, 0),
    "into_inputs": (3000, 40, 12000, 4, 0, 0.0, 25),
}


def levels_small():
    """RecomputeLevels + SortConnectionsByLevel through the reference's own
    Topological constructor, on the level_graph cases above."""
    out = {}
    for name, (nu, ni, nc, seed, back, dfrac, into) in LEVEL_CASES.items():
        f, t, d = workloads.level_graph(nu, ni, nc, seed, back_edges=back, dead_frac=dfrac,
                                        into_inputs=into)
        lv, fo, to, so, do = oracle.ref_levels_run(nu, ni, f, t, d)
        out.update({f"{name}_params": np.array([nu, ni, nc, seed, back, into], np.int64),
                    f"{name}_dead_frac": np.float64(dfrac), f"{name}_level": lv,
                    f"{name}_from": fo, f"{name}_to": to, f"{name}_src_level": so,
                    f"{name}_dead": do})
    np.savez_compressed(HERE / "levels_small.npz", **out)


def structural_net():
    """The structural test policies (oracle/structural_policies.hpp) through the
    reference's own Topological Network: the small case whole, the medium case
    as sizes and SHA-256 digests of each array."""
    import hashlib
    out = {}
    for name in ("small", "medium"):
        variant, n_in, h1, h2, seed, steps, cap = oracle.STRUCTURAL_CASES[name]
        r = oracle.ref_structural_run(name)
        out[f"{name}_params"] = np.array([variant, n_in, h1, h2, seed, steps], np.int64)
        out[f"{name}_inputs"] = oracle.structural_inputs(name)
        for k, v in r.items():
            v = np.ascontiguousarray(v).reshape(-1)
            if name == "small":
                out[f"{name}_{k}"] = v
            else:
                out[f"{name}_{k}_size"] = np.int64(v.size)
                out[f"{name}_{k}_sha256"] = np.array(hashlib.sha256(v.tobytes()).hexdigest())
    np.savez_compressed(HERE / "structural_net.npz", **out)


if __name__ == "__main__":
    ob.build()
    if oracle.ref() is None:
        sys.exit("reference build missing: the reference tree is needed to make fixtures")
    makers = {"sweep_hebbian_small": sweep_hebbian_small, "swifttd_small": swifttd_small,
              "mlp_xor_small": mlp_xor_small, "ipc_small": ipc_small,
              "levels_small": levels_small, "structural_net": structural_net}
    for name in sys.argv[1:] or list(makers):  # names given: only those fixtures
        makers[name]()
    print("fixtures written to", HERE)
