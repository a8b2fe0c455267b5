"""Build recipe for the sm_100a shared library ``libplastix_b200.so``.

Compiles every ``csrc/*.cu`` with nvcc for sm_100a only (no other targets,
no PTX JIT fallback) and links them into ``plastix_b200/libplastix_b200.so``
in the source tree. ``--fmad=false`` keeps every multiply and add separately
rounded, as the reference's x86-64 build does, so the per-row sums and
per-connection updates can match it bit for bit.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libplastix_b200.so"
# Measurement-only kernels (the benchmark's sweep-ceiling probes) live in a
# library of their own so that the product library carries none of them.
PROBE_SRC = PKG / "probe" / "probe.cu"
PROBE_LIB = PKG / "libplastix_probe.so"
# Programs written against the reference's C++ API (include/plastix/*.hpp).
APPS = {"network_sweep": PKG / "apps" / "network_sweep.cu",
        "xor_train": PKG / "apps" / "xor_train.cu"}
APP_FLAGS = ["-std=c++20", "--expt-relaxed-constexpr", "-O2", "--fmad=false", "-lineinfo",
             "-diag-suppress=20050", f"-I{ROOT / 'include'}"]


def app_path(name: str) -> Path:
    return OBJ / name
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_probe(verbose)
    for name in APPS:
        build_app(name)
    return LIB


def build_app(name: str) -> Path:
    exe = app_path(name)
    deps = [APPS[name], LIB] + sorted((ROOT / "include").rglob("*.h*"))
    if _stale(exe, deps):
        cmd = [NVCC, *ARCH, *APP_FLAGS, str(APPS[name]), "-o", str(exe), f"-L{PKG}",
               "-lplastix_b200", "-Xlinker", "-rpath=$ORIGIN/.."]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {name}:\n{r.stdout}\n{r.stderr}")
    return exe


def build_probe(verbose: bool = False) -> Path:
    """libplastix_probe.so: the sweep-ceiling measurement kernels, linked
    against the product library (it uses its context and error reporting)."""
    obj = _compile(PROBE_SRC, verbose)
    if _stale(PROBE_LIB, [obj, LIB]):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(PROBE_LIB), str(obj), f"-L{PKG}",
               "-lplastix_b200", "-Xlinker", "-rpath=$ORIGIN", "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"probe link failed:\n{r.stdout}\n{r.stderr}")
    return PROBE_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
