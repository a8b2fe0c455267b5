"""The single-layer sweep written against the reference's C++ API
(plastix::Network<Traits> with PLASTIX_HD policies, stepped with DoStep:
plastix_b200/apps/network_sweep.cu) against the oracle, bit for bit: the
destination-major forward accumulation (Map on consecutive connections per
lane, each unit's values combined in connection order) and the
per-connection Hebbian trace update, for short, long and empty rows. Both
spellings of the rule run: a user hook (generic device passes) and the
library's HebbianTraceUpdate policy (one fused sliced sweep per DoStep)."""
import subprocess

import numpy as np
import pytest

from plastix_b200 import build, workloads


def _write_layer(path, L):
    with open(path, "wb") as f:
        np.array([L.n_src, L.n_dst, L.from_id.size], np.uint64).tofile(f)
        np.ascontiguousarray(L.from_id, np.uint32).tofile(f)
        np.ascontiguousarray(L.to_id - L.n_src, np.uint32).tofile(f)
        np.ascontiguousarray(L.weight, np.float32).tofile(f)
        np.ascontiguousarray(L.act_in, np.float32).tofile(f)


def test_api_program_is_built():
    exe = build.build_app("network_sweep")
    assert exe.exists()


@pytest.mark.gpu
@pytest.mark.parametrize("traits", ["generic", "fused"])
@pytest.mark.parametrize("case", ["random", "rows"])
def test_api_sweep_matches_oracle(tmp_path, orc, case, traits):
    if case == "random":
        L = workloads.sparse_layer(20000, 3000, 200003, seed=17)
    else:
        L = workloads.sparse_layer_rows(900, [0, 5, 300, 0, 1, 2000, 64, 65, 257] * 40, seed=5)
    _write_layer(tmp_path / "layer.bin", L)
    exe = build.build_app("network_sweep")
    r = subprocess.run([str(exe), "check", str(tmp_path), "3", traits], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, L.n_src, 0.9, 1e-3,
                               sweeps=3)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "out.bin", np.float32), a[L.n_src:])
    np.testing.assert_array_equal(np.fromfile(tmp_path / "w.bin", np.float32), w)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "e.bin", np.float32), e)


@pytest.mark.gpu
@pytest.mark.parametrize("traits", ["generic", "fused"])
def test_api_host_edits_between_steps(tmp_path, orc, traits):
    """Weights written, connections killed and traces read on the host
    between DoSteps: the fused route's slot-order copies are unpacked for the
    read and re-packed (with the dead-aware kernel) after the writes, so every
    step still matches the oracle bit for bit."""
    L = workloads.sparse_layer_rows(700, [0, 3, 150, 1, 900, 33] * 50, seed=11)
    _write_layer(tmp_path / "layer.bin", L)
    exe = build.build_app("network_sweep")
    r = subprocess.run([str(exe), "check-edit", str(tmp_path), "3", traits], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    n = L.from_id.size
    act = np.concatenate([L.act_in, np.zeros(L.n_dst, np.float32)])
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace, act, L.n_src, 0.9, 1e-3,
                               sweeps=1)
    w = w.copy()
    w[0] = np.float32(w[0] + np.float32(0.25))
    w[n // 2] = np.float32(w[n // 2] - np.float32(0.5))
    dead = np.zeros(n, np.uint8)
    dead[[n // 5, n // 7]] = 1
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, w, e, a, L.n_src, 0.9, 1e-3, sweeps=2,
                               dead=dead)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "out.bin", np.float32), a[L.n_src:])
    np.testing.assert_array_equal(np.fromfile(tmp_path / "w.bin", np.float32), w)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "e.bin", np.float32), e)
