"""The device Network<Traits> (include/plastix/plastix.hpp): C++ programs
whose policies carry PLASTIX_HD and run on the GPU through the same API as
the reference header library, against the reference-made fixtures:

* network_xor.cu -- the XOR MLP (Topological, sigmoid, MSE, backward,
  gradient descent): initial weights bit for bit (same host generator as the
  reference's RandomUniformWeight), weights and predictions after 200 epochs
  at 1e-5 relative (device expf against the host's).
* network_ipc.cu -- 30 streaming-iPC steps (Pipeline, tanh): weights, value
  nodes and errors at 1e-5 relative.
* network_swifttd.cu -- 200 SwiftTD steps (per-connection hooks that add
  into the globals, run with the sequential connection update): V per step,
  weights and log step sizes at 1e-5 relative.
* network_structural.cu -- the structural policies of
  oracle/structural_policies.hpp (unit and connection pruning, hash-chosen
  connection proposals, commit with InitConnection, Topological re-sort with
  RecomputeLevels) on a small and a medium network: every output, connection
  field and unit level bit for bit (the medium case through digests).
* network_mse_fusion.cu -- the library MSELoss fused into the forward
  Apply (Pipeline DoStep) and run per output in parallel, against a user
  loss with the same body: bit for bit.

On the CPU the programs are compiled (nvcc cross-compiles for sm_100a)."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
NVCC = "/usr/local/cuda/bin/nvcc"


def compile_prog(name: str, out: Path) -> Path:
    exe = out / name
    lib = ROOT / "plastix_b200"
    cmd = [NVCC, "-std=c++20", "--expt-relaxed-constexpr", "-gencode",
           "arch=compute_100a,code=sm_100a", "-O2", "--fmad=false", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "cpp" / f"{name}.cu"), "-o", str(exe),
           f"-L{lib}", "-lplastix_b200", f"-Xlinker=-rpath,{lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc failed:\n{r.stdout}\n{r.stderr}")
    return exe


def parse(out: str):
    vals = {}
    for line in out.splitlines():
        k, v = line.split()
        vals.setdefault(k, []).append(float.fromhex(v))
    return {k: np.array(v, np.float32) for k, v in vals.items()}


@pytest.mark.parametrize("name", ["network_xor", "network_ipc", "network_swifttd",
                                  "network_structural", "network_mse_fusion"])
def test_device_network_programs_compile(tmp_path, name):
    assert compile_prog(name, tmp_path).exists()


@pytest.mark.gpu
def test_mse_loss_in_apply_epilogue_equals_user_loss(tmp_path):
    """plastix::MSELoss run in the forward Apply epilogue (Pipeline DoStep)
    or as a parallel kernel (DoCalculateLoss, Topological DoStep) leaves the
    network bit for bit where a user loss with the same body (the generic
    one-thread loss hook) leaves it."""
    exe = compile_prog("network_mse_fusion", tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip() == "ok"


@pytest.mark.gpu
def test_device_network_xor_matches_reference(tmp_path):
    z = np.load(GOLDEN / "mlp_xor_small.npz")
    exe = compile_prog("network_xor", tmp_path)
    r = subprocess.run([str(exe), "200"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    v = parse(r.stdout)
    np.testing.assert_array_equal(v["w0"].view(np.uint32), z["w_init"].view(np.uint32))
    np.testing.assert_allclose(v["w"], z["w_200"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v["p"], z["preds_200"], rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_device_network_ipc_matches_reference(tmp_path):
    z = np.load(GOLDEN / "ipc_small.npz")
    for k in ("w0", "x0", "inputs", "targets"):
        np.ascontiguousarray(z[k], np.float32).tofile(tmp_path / f"{k}.bin")
    exe = compile_prog("network_ipc", tmp_path)
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    v = parse(r.stdout)
    np.testing.assert_allclose(v["w"], z["w"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v["x"], z["x"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v["e"], z["err"], rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_device_network_swifttd_matches_reference(tmp_path):
    z = np.load(GOLDEN / "swifttd_small.npz")
    np.ascontiguousarray(z["features"], np.float32).tofile(tmp_path / "features.bin")
    np.ascontiguousarray(z["rewards"], np.float32).tofile(tmp_path / "rewards.bin")
    exe = compile_prog("network_swifttd", tmp_path)
    r = subprocess.run([str(exe), str(tmp_path), str(int(z["n"]))], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    v = parse(r.stdout)
    np.testing.assert_allclose(v["v"], z["v"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v["w"], z["fields"][0], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(v["b"], z["fields"][9], rtol=1e-5, atol=1e-6)


def _run_structural(tmp_path, name, resume_at=None, on_device=False):
    z = np.load(GOLDEN / "structural_net.npz")
    variant, n_in, h1, h2, seed, steps = (int(v) for v in z[f"{name}_params"])
    variant += 2 if on_device else 0
    np.ascontiguousarray(z[f"{name}_inputs"], np.float32).tofile(tmp_path / "inputs.bin")
    exe = compile_prog("network_structural", tmp_path)
    args = [str(exe), str(variant), str(n_in), str(h1), str(h2), str(seed), str(steps),
            str(tmp_path)] + ([] if resume_at is None else [str(resume_at)])
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    types = {"outputs": np.float32, "from": np.uint32, "to": np.uint32, "dead": np.uint8,
             "src_level": np.uint16, "w": np.float32, "level": np.uint16, "act": np.float32}
    got = {k: np.fromfile(tmp_path / f"{k}.bin", dtype=t) for k, t in types.items()}
    return z, got


@pytest.mark.gpu
@pytest.mark.parametrize("on_device", [False, True], ids=["host-decisions", "device-decisions"])
@pytest.mark.parametrize("resume_at", [None, 2, 4])
def test_device_network_structural_small_matches_reference(tmp_path, resume_at, on_device):
    """Two-way proposals (into input units, cycles), a unit pruned at step 2,
    weights pruned below 0.02: five steps, every array bit for bit -- also
    when the run is checkpointed before step `resume_at` and resumed in a
    newly built network (Save / Load); with the structural decisions made on
    the host copy (the default) and on the device (DeviceStructure)."""
    z, got = _run_structural(tmp_path, "small", resume_at, on_device)
    for k, v in got.items():
        want = z[f"small_{k}"].reshape(-1)
        assert v.size == want.size, k
        np.testing.assert_array_equal(v.view(np.uint8), want.view(np.uint8), err_msg=k)


@pytest.mark.gpu
@pytest.mark.parametrize("on_device", [False, True], ids=["host-decisions", "device-decisions"])
@pytest.mark.parametrize("resume_at", [None, 1])
def test_device_network_structural_medium_matches_reference(tmp_path, resume_at, on_device):
    """32 -> 200 -> 50 with forward proposals over ~60k unit pairs per step
    (on the device the parallel enumeration runs over many chunks): digests
    of every array, straight through and resumed from a checkpoint."""
    import hashlib
    z, got = _run_structural(tmp_path, "medium", resume_at, on_device)
    for k, v in got.items():
        assert v.size == int(z[f"medium_{k}_size"]), k
        assert hashlib.sha256(v.tobytes()).hexdigest() == str(z[f"medium_{k}_sha256"]), k
