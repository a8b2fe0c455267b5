"""The C++ host layer (include/plastix_b200.hpp): a C++ program with no
Python in its path builds and steps the single-layer trace network and the
SwiftTD network through the C ABI. On the CPU the program is compiled (the
header and the library's exports link); on the GPU its results are compared
with the oracle -- bit for bit for the sweep (rows <= 256), 1e-5 relative for
SwiftTD (double-precision sums on the device)."""
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "cpp" / "host_networks.cpp"
LIBDIR = ROOT / "plastix_b200"
CUDA = Path("/usr/local/cuda")


def build(out: Path) -> Path:
    from plastix_b200 import _abi
    _abi.lib()  # the library must exist (built by __graft_entry__.build)
    exe = out / "host_networks"
    cmd = ["g++", "-std=c++20", "-O2", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           str(SRC), f"-L{LIBDIR}", "-lplastix_b200", f"-L{CUDA / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_host_program_compiles_and_links(tmp_path):
    exe = build(tmp_path)
    assert exe.exists() and os.access(exe, os.X_OK)


@pytest.mark.gpu
def test_cpp_host_program_matches_oracle(tmp_path, orc):
    from plastix_b200 import workloads
    exe = build(tmp_path)
    n_src, n_dst, n, sweeps = 3000, 2000, 120_000, 3
    L = workloads.sparse_layer(n_src, n_dst, n, seed=77)
    for name, arr in (("from", L.from_id), ("to", L.to_id), ("w", L.weight),
                      ("act", L.act_in)):
        np.ascontiguousarray(arr).tofile(tmp_path / f"in_{name}.bin")
    td_n, td_steps = 5000, 12
    rng = np.random.default_rng(78)
    sets = [np.sort(rng.choice(td_n, 50, replace=False)).astype(np.uint32)
            for _ in range(td_steps)]
    offs = np.concatenate([[0], np.cumsum([s.size for s in sets])]).astype(np.uint32)
    rewards = rng.normal(size=td_steps).astype(np.float32)
    offs.tofile(tmp_path / "in_td_offs.bin")
    np.concatenate(sets).tofile(tmp_path / "in_td_idx.bin")
    rewards.tofile(tmp_path / "in_td_rw.bin")
    r = subprocess.run([str(exe), str(tmp_path), str(n_src), str(n_dst), str(n), str(sweeps),
                        str(td_n), str(td_steps)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    w, e, a = orc.step_hebbian(L.from_id, L.to_id, L.weight, L.trace,
                               np.concatenate([L.act_in, np.zeros(n_dst, np.float32)]), n_src,
                               0.9, 1e-3, sweeps=sweeps)
    got = lambda name, dt: np.fromfile(tmp_path / f"out_{name}.bin", dtype=dt)  # noqa: E731
    np.testing.assert_array_equal(got("act", np.uint32), a[n_src:].view(np.uint32))
    np.testing.assert_array_equal(got("w", np.uint32), w.view(np.uint32))
    np.testing.assert_array_equal(got("e", np.uint32), e.view(np.uint32))
    fields = orc.td_fields(td_n)
    g = orc.td_globals(gamma=0.99)
    vs = []
    for s in range(td_steps):
        f = np.zeros(td_n, np.float32)
        f[sets[s]] = 1.0
        vs.append(orc.swifttd_step(fields, f, rewards[s], g, True))
    np.testing.assert_allclose(got("td_v", np.float32), np.array(vs, np.float32), rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(got("td_w", np.float32), fields[0], rtol=1e-5, atol=1e-6)
