"""Build recipe (TEST INFRASTRUCTURE ONLY): the reference's own examples and
unit tests compiled against this repository's device headers.

Reads from the reference checkout ($PLX_REFERENCE_ROOT, else ``reference``
beside this repository) -- only in the build container; the GPU machines use
the prebuilt binaries:

* ``examples/*/*.cpp`` (the nine example programs), each built into
  ``tests/refsuite/_build/examples/<name>``;
* ``tests/test_plastix.cpp``, ``test_plastix_pipeline.cpp``,
  ``test_alloc.cpp`` and ``test_soa.cpp`` (with ``test_soa_fields.inc``),
  each built with the minimal googletest-compatible harness of
  ``tests/refsuite/gtest`` into ``tests/refsuite/_build/tests/<name>``.

The one change to those sources is the annotation the device API asks for:
``PLASTIX_HD`` in front of every static member function of a struct (the
policy hooks, which run in kernels) and of every free function such a member
calls (helpers like the iPC example's ``Act``), except functions that name
host-only state -- a host stream (the imprinting learner's InitUnit and
connection helper) or a non-constant static data member (a unit test's
pruning predicate) -- which device code cannot name; the device API runs
those hooks (AddUnit, and by default PruneUnit and AddConn) on the host.
Nothing else is edited. The
annotated copies and the binaries live in ``tests/refsuite/_build/``
(git-ignored; they travel to the GPU machines with the working tree).

Each example is also built unchanged with g++ from the reference sources
(``oracle/_ref/examples/<name>``, the reference's own CPU path) -- that is
what ``tests/golden/make_reference_outputs.py`` runs to record the outputs
the GPU builds are compared with.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF_ROOT = Path(os.environ.get("PLX_REFERENCE_ROOT", ROOT.parent / "reference"))
OUT = HERE / "_build"
REF_OUT = ROOT / "oracle" / "_ref" / "examples"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
LIB_DIR = ROOT / "plastix_b200"

EXAMPLES = ["fcc-nn", "imprinting-learner", "ipc-linear", "ipc-multilayer", "linear-regression",
            "manual-fcc", "mlp-xor", "pipeline-fcc", "swifttd"]
UNIT_TESTS = ["test_plastix", "test_plastix_pipeline", "test_alloc", "test_soa"]
# TEST cases per file in the reference (tests/CMakeLists.txt builds them into
# one binary); the GPU test checks that every one of them ran and passed.
UNIT_TEST_COUNTS = {"test_plastix": 55, "test_plastix_pipeline": 38, "test_alloc": 3,
                    "test_soa": 5}

NVCC_FLAGS = ["-std=c++20", "--expt-relaxed-constexpr", "-gencode",
              "arch=compute_100a,code=sm_100a", "-O2", "--fmad=false", "-w",
              "-diag-suppress=20050"]


def example_name(d: str) -> str:
    return d.replace("-", "_")


# ---------------------------------------------------------------------------
# annotation
# ---------------------------------------------------------------------------
_MEMBER_FN = re.compile(r"^(\s+)(static\s+(?!constexpr\b|inline\s+constexpr\b)[^;=(]*?\b\w+\s*\()")
_FREE_FN = re.compile(r"^((?:inline\s+|static\s+)*)((?:[\w:]+(?:<[^>]*>)?\s*[*&]?\s+)+)(\w+)\s*\(")


def _struct_bodies(lines):
    """Index ranges [start, end) of struct definitions that are not nested in
    another struct (at namespace scope, any namespace depth)."""
    out = []
    depth = 0
    start = start_depth = None
    for i, line in enumerate(lines):
        code = line.split("//")[0]
        if start is None and re.match(r"^\s*struct\s+\w+[^;]*\{", code):
            start, start_depth = i, depth
        depth += code.count("{") - code.count("}")
        if start is not None and depth == start_depth:
            out.append((start, i + 1))
            start = None
    return out


def _body(lines, i):
    """The text of the function whose signature starts on line i."""
    depth, seen, out = 0, False, []
    for line in lines[i:]:
        code = line.split("//")[0]
        out.append(code)
        depth += code.count("{") - code.count("}")
        seen = seen or "{" in code
        if seen and depth <= 0:
            break
        if not seen and code.rstrip().endswith(";"):
            break
    return "\n".join(out)


_HOST_ONLY = ("std::cout", "std::cerr", "std::clog")
_STATIC_DATA = re.compile(r"^\s+static\s+(?!constexpr\b)[\w:<>\s]+?\b(\w+)\s*;")


def annotate(text: str) -> str:
    """PLASTIX_HD before every static member function of a (top-level) struct
    and before every free function that one of them calls -- except those
    that write to a host stream (std::cout, ...), which device code cannot
    name, nor those naming a non-constant static data member (a host
    variable); the device API runs such hooks (AddUnit, and by default
    PruneUnit and AddConn) on the host, where they need no annotation."""
    lines = text.split("\n")
    bodies = _struct_bodies(lines)
    in_struct = set()
    called = set()
    for a, b in bodies:
        for i in range(a, b):
            in_struct.add(i)
            called.update(re.findall(r"\b(\w+)\s*\(", lines[i]))
    # non-constant static data members: host variables device code cannot name
    statics = set()
    for i in in_struct:
        m = _STATIC_DATA.match(lines[i])
        if m:
            statics.add(m.group(1))
    host_only = _HOST_ONLY + tuple(statics)
    for i in sorted(in_struct):
        m = _MEMBER_FN.match(lines[i])
        if m and "PLASTIX_HD" not in lines[i]:
            if any(re.search(rf"\b{re.escape(h)}\b", _body(lines, i)) for h in host_only):
                continue
            lines[i] = m.group(1) + "PLASTIX_HD " + lines[i][len(m.group(1)):]
    for i, line in enumerate(lines):
        if i in in_struct or line.startswith((" ", "\t", "#", "//")):
            continue
        m = _FREE_FN.match(line)
        if not m or m.group(3) == "main" or m.group(3) not in called:
            continue
        if "PLASTIX_HD" in line or line.rstrip().endswith(";"):
            continue
        if any(h in _body(lines, i) for h in _HOST_ONLY):
            continue
        lines[i] = "PLASTIX_HD " + line
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# builds
# ---------------------------------------------------------------------------
def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"build failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).exists() and Path(d).stat().st_mtime > t for d in deps)


def _headers():
    return sorted((ROOT / "include").rglob("*.h*")) + [LIB_DIR / "libplastix_b200.so",
                                                       Path(__file__)]


def _device_link():
    return [f"-I{ROOT / 'include'}", f"-L{LIB_DIR}", "-lplastix_b200",
            f"-Xlinker=-rpath,{LIB_DIR}"]


def build_example(d: str) -> Path:
    name = example_name(d)
    src = REF_ROOT / "examples" / d / f"{name}.cpp"
    work = OUT / "src" / "examples"
    work.mkdir(parents=True, exist_ok=True)
    patched = work / f"{name}.cu"
    exe = OUT / "examples" / name
    exe.parent.mkdir(parents=True, exist_ok=True)
    if _stale(exe, [src] + _headers()):
        patched.write_text(annotate(src.read_text()))
        _run([NVCC, *NVCC_FLAGS, str(patched), "-o", str(exe), *_device_link()])
    return exe


def build_reference_example(d: str) -> Path:
    """The unchanged example on the reference's own CPU path (g++, the
    reference headers), for recording the outputs to compare with."""
    name = example_name(d)
    src = REF_ROOT / "examples" / d / f"{name}.cpp"
    exe = REF_OUT / name
    exe.parent.mkdir(parents=True, exist_ok=True)
    deps = [src, Path(__file__)] + sorted((REF_ROOT / "include" / "plastix").glob("*.hpp"))
    if _stale(exe, deps):
        _run(["g++", "-std=c++20", "-O2", f"-I{REF_ROOT / 'include'}", str(src),
              str(REF_ROOT / "src" / "plastix.cpp"), "-o", str(exe)])
    return exe


def build_unit_test(name: str) -> Path:
    src = REF_ROOT / "tests" / f"{name}.cpp"
    work = OUT / "src" / "tests"
    work.mkdir(parents=True, exist_ok=True)
    patched = work / f"{name}.cu"
    extra = []
    inc = REF_ROOT / "tests" / "test_soa_fields.inc"
    if name == "test_soa":
        (work / inc.name).write_text(inc.read_text())
        extra = [inc]
    exe = OUT / "tests" / name
    exe.parent.mkdir(parents=True, exist_ok=True)
    if _stale(exe, [src, HERE / "gtest" / "gtest.h", HERE / "gtest_main.cpp"] + extra + _headers()):
        patched.write_text(annotate(src.read_text()))
        _run([NVCC, *NVCC_FLAGS, f"-I{HERE}", f"-I{work}", str(patched), "-x", "cu",
              str(HERE / "gtest_main.cpp"), "-o", str(exe), *_device_link()])
    return exe


def available() -> bool:
    return (REF_ROOT / "examples").is_dir() and (REF_ROOT / "tests").is_dir()


def build(jobs: int | None = None) -> list[Path]:
    """Builds every example and unit-test binary (a no-op without the
    reference tree: the prebuilt binaries are used as they are)."""
    if not available():
        return []
    jobs = jobs or min(8, os.cpu_count() or 1)
    tasks = ([(build_example, d) for d in EXAMPLES] + [(build_reference_example, d)
                                                        for d in EXAMPLES]
             + [(build_unit_test, t) for t in UNIT_TESTS])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        return list(ex.map(lambda t: t[0](t[1]), tasks))


if __name__ == "__main__":
    for p in build():
        print(p)
    sys.exit(0)
