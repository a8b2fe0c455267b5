"""Build recipe for the oracle (test infrastructure only).

* ``oracle/libplx_oracle.so`` — the C restatement (plx_oracle.c), built with
  the reference's arithmetic settings: x86-64 SSE, ``-O2``,
  ``-ffp-contract=off`` (no fused multiply-add), like the reference's own
  ``-std=c++20 -O2`` build.
* ``oracle/_ref/libplx_ref.so`` — the reference itself: its headers
  compiled from the reference tree (``$PLX_REFERENCE_ROOT/include``, by
  default ``../reference`` beside this repository) together with
  ``oracle/ref_harness.cpp``, ``oracle/ref_mlp.cpp`` and ``oracle/ref_ipc.cpp``,
  which compile the reference's ``examples/swifttd/swifttd.cpp``,
  ``examples/mlp-xor/mlp_xor.cpp`` and ``examples/ipc-multilayer/ipc_multilayer.cpp``
  unchanged (each ``main`` renamed) to drive their own policies. Only when the reference tree is present (it is
  not on the GPU machines, which use the prebuilt file). The one change to the
  reference sources: the fixed capacities ``UnitAlloc(4096), ConnAlloc(4096 *
  4)`` of ``include/plastix/plastix.hpp`` become calls into the harness, so
  networks of the benchmark sizes fit. The patched header copy lives in a
  temporary directory and is deleted after the build.
* ``oracle/_ref/xor_train`` — ``plastix_b200/apps/xor_train.cu`` (the XOR
  training run) built with g++ against the unchanged reference headers.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
# The reference checkout: PLX_REFERENCE_ROOT, else a `reference` directory
# beside this repository's root.
REF_ROOT = Path(os.environ.get("PLX_REFERENCE_ROOT", HERE.parents[1] / "reference"))
ORACLE_SO = HERE / "libplx_oracle.so"
REF_DIR = HERE / "_ref"
REF_SO = REF_DIR / "libplx_ref.so"

CAPACITY_LITERAL = "UnitAlloc(4096), ConnAlloc(4096 * 4)"
CAPACITY_PATCH = "UnitAlloc(::plx_ref_unit_capacity()), ConnAlloc(::plx_ref_conn_capacity())"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build_oracle() -> Path:
    src = HERE / "plx_oracle.c"
    if _stale(ORACLE_SO, [src, Path(__file__)]):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11",
               "-Wall", str(src), "-o", str(ORACLE_SO), "-lm"]
        subprocess.run(cmd, check=True)
    return ORACLE_SO


def build_reference() -> Path | None:
    """Compile the reference from its own tree; None when it is absent."""
    hpp = REF_ROOT / "include" / "plastix" / "plastix.hpp"
    if not hpp.exists():
        return REF_SO if REF_SO.exists() else None
    harness = HERE / "ref_harness.cpp"
    units = [harness, HERE / "ref_mlp.cpp", HERE / "ref_ipc.cpp"]
    examples = [REF_ROOT / "examples" / d for d in ("swifttd", "mlp-xor", "ipc-multilayer")]
    deps = (units + [Path(__file__)] + [e / f"{e.name.replace('-', '_')}.cpp" for e in examples]
            + sorted((REF_ROOT / "include" / "plastix").glob("*.hpp")))
    if not _stale(REF_SO, deps):
        return REF_SO
    REF_DIR.mkdir(exist_ok=True)
    with tempfile.TemporaryDirectory(prefix="plx_ref_") as tmp:
        inc = Path(tmp) / "include"
        shutil.copytree(REF_ROOT / "include", inc)
        text = (inc / "plastix" / "plastix.hpp").read_text()
        if text.count(CAPACITY_LITERAL) != 1:
            raise RuntimeError("reference plastix.hpp no longer has the capacity "
                               f"literal {CAPACITY_LITERAL!r}; update the recipe")
        (inc / "plastix" / "plastix.hpp").write_text(
            text.replace(CAPACITY_LITERAL, CAPACITY_PATCH))
        prelude = Path(tmp) / "plx_ref_capacity.h"
        prelude.write_text("#include <cstddef>\n"
                           "std::size_t plx_ref_unit_capacity();\n"
                           "std::size_t plx_ref_conn_capacity();\n")
        cmd = (["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-pthread",
                "-include", str(prelude), f"-I{inc}"] + [f"-I{e}" for e in examples]
               + [str(u) for u in units] + [
               str(REF_ROOT / "src" / "plastix.cpp"), "-o", str(REF_SO)])
        subprocess.run(cmd, check=True)
    return REF_SO


XOR_SRC = HERE.parent / "plastix_b200" / "apps" / "xor_train.cu"
REF_XOR = REF_DIR / "xor_train"


def build_reference_xor() -> Path | None:
    """``oracle/_ref/xor_train``: the XOR training program of
    ``plastix_b200/apps/xor_train.cu`` compiled with g++ against the
    reference's own, unchanged headers (and ``src/plastix.cpp``) -- the
    reference's CPU implementation of that run, the benchmark's baseline."""
    hpp = REF_ROOT / "include" / "plastix" / "plastix.hpp"
    if not hpp.exists():
        return REF_XOR if REF_XOR.exists() else None
    deps = [XOR_SRC, Path(__file__)] + sorted((REF_ROOT / "include" / "plastix").glob("*.hpp"))
    if _stale(REF_XOR, deps):
        REF_DIR.mkdir(exist_ok=True)
        cmd = ["g++", "-std=c++20", "-O2", "-x", "c++", f"-I{REF_ROOT / 'include'}",
               str(XOR_SRC), "-x", "none", str(REF_ROOT / "src" / "plastix.cpp"), "-o",
               str(REF_XOR)]
        subprocess.run(cmd, check=True)
    return REF_XOR


def build() -> None:
    build_oracle()
    build_reference()
    build_reference_xor()


if __name__ == "__main__":
    build()
    print(ORACLE_SO, REF_SO if REF_SO.exists() else "(reference not built)")
    sys.exit(0)
