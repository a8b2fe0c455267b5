"""The reference's own programs on the device path: its nine examples and
its four unit-test files (101 TEST cases), built unchanged except for the
PLASTIX_HD annotations against this repository's device headers
(tests/refsuite/build.py), run on the GPU.

* Examples: the exit code must equal the reference's (mlp_xor,
  linear_regression and ipc_multilayer decide PASS/FAIL by it), every line's
  text must equal the reference's, and every printed number must match the
  reference's CPU output (tests/golden/reference_examples.json, recorded by
  tests/golden/make_reference_outputs.py) within two units of its last
  printed digit -- the device evaluates exp/tanh/log with CUDA's functions,
  not glibc's, and the runs are thousands of learning steps long.
* Unit tests: every TEST case of each file runs and passes under the
  googletest-compatible harness (tests/refsuite/gtest); the allocator and
  SoA-macro files need no GPU and also run in the CPU suite.
"""
import importlib.util
import json
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
_spec = importlib.util.spec_from_file_location("plx_refsuite_build",
                                               ROOT / "tests" / "refsuite" / "build.py")
refsuite = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(refsuite)

GOLDEN = json.loads((ROOT / "tests" / "golden" / "reference_examples.json").read_text())
BUILD = refsuite.OUT
HOST_ONLY_TESTS = ("test_alloc", "test_soa")  # allocator / macros: no device work

_NUM = re.compile(r"(-?\d+(?:\.\d+)?(?:[eE][-+]?\d+)?)")


def _binary(kind: str, name: str) -> Path:
    exe = BUILD / kind / name
    if not exe.exists():
        if refsuite.available():
            refsuite.build()
        if not exe.exists():
            pytest.skip(f"{exe} was not built (no reference tree at build time)")
    return exe


def _split(line: str):
    parts = _NUM.split(line)
    text = "".join(p for i, p in enumerate(parts) if i % 2 == 0)
    nums = [p for i, p in enumerate(parts) if i % 2 == 1]
    return re.sub(r"\s+", "", text), nums


def _ulp(s: str) -> float:
    """One unit of the last printed digit of a decimal string (integers, such
    as step counts and state ids, must match exactly)."""
    return 10.0 ** -len(s.split(".")[1]) if "." in s else 0.0


def compare_outputs(got: str, want: str, units: float = 2.0):
    """Mismatches between two example outputs: lines and text must be equal,
    decimal numbers equal within `units` of their last printed digit."""
    g, w = got.rstrip("\n").splitlines(), want.rstrip("\n").splitlines()
    if len(g) != len(w):
        return [f"{len(g)} lines, want {len(w)}"]
    bad = []
    for i, (a, b) in enumerate(zip(g, w)):
        ta, na = _split(a)
        tb, nb = _split(b)
        if ta != tb or len(na) != len(nb):
            bad.append(f"line {i + 1}: {a!r} vs {b!r}")
            continue
        for x, y in zip(na, nb):
            if abs(float(x) - float(y)) > units * _ulp(y) * (1 + 1e-9):
                bad.append(f"line {i + 1}: {x} vs {y} ({a!r})")
    return bad


def test_output_comparison_rules():
    want = "Epoch     0  loss: 1.2345\nPASS\n"
    assert compare_outputs("Epoch     0  loss: 1.2346\nPASS\n", want) == []
    assert compare_outputs("Epoch     0  loss: 1.2349\nPASS\n", want)
    assert compare_outputs("Epoch     1  loss: 1.2345\nPASS\n", want)
    assert compare_outputs("Epoch     0  loss: 1.2345\nFAIL\n", want)


def test_annotation_marks_device_hooks_only():
    src = "\n".join([
        "namespace {",
        "struct P {",
        "  static size_t Target;",
        "  static float Map(auto &U, size_t, size_t S, auto &C, size_t Id, auto &) {",
        "    return Helper(1.0f);",
        "  }",
        "  static bool ShouldPrune(auto &, size_t Id, auto &) { return Id == Target; }",
        "  static void Init(auto &, size_t) { std::cout << 1; }",
        "  static constexpr float Rate = 0.5f;",
        "};",
        "float Helper(float x) { return x; }",
        "void HostOnly(int) {}",
        "}",
    ])
    out = refsuite.annotate(src).splitlines()
    assert out[3].startswith("  PLASTIX_HD static float Map")
    assert "PLASTIX_HD" not in out[2] and "PLASTIX_HD" not in out[8]
    assert "PLASTIX_HD" not in out[6]  # names a static data member
    assert "PLASTIX_HD" not in out[7]  # writes to a host stream
    assert out[10].startswith("PLASTIX_HD float Helper")
    assert "PLASTIX_HD" not in out[11]


@pytest.mark.parametrize("name", HOST_ONLY_TESTS)
def test_reference_unit_tests_on_host_storage(name):
    exe = _binary("tests", name)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout[-3000:]
    assert r.stdout.count("[       OK ]") == refsuite.UNIT_TEST_COUNTS[name], r.stdout[-2000:]


@pytest.mark.gpu
@pytest.mark.parametrize("name", refsuite.UNIT_TESTS)
def test_reference_unit_tests_on_device(name):
    exe = _binary("tests", name)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    failed = [l for l in r.stdout.splitlines() if l.startswith("[  FAILED  ]")]
    assert r.returncode == 0, "\n".join(failed) + "\n" + r.stdout[-4000:] + r.stderr[-2000:]
    assert r.stdout.count("[       OK ]") == refsuite.UNIT_TEST_COUNTS[name], r.stdout[-2000:]


@pytest.mark.gpu
@pytest.mark.parametrize("name", [refsuite.example_name(d) for d in refsuite.EXAMPLES])
def test_reference_example_on_device(name):
    exe = _binary("examples", name)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900)
    want = GOLDEN[name]
    assert r.returncode == want["returncode"], r.stdout[-2000:] + r.stderr[-2000:]
    bad = compare_outputs(r.stdout, want["stdout"])
    assert not bad, "\n".join(bad[:20]) + "\n--- got ---\n" + r.stdout[-3000:]
