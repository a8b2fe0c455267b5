"""Records the outputs of the reference's nine example programs run on the
reference's own CPU path (TEST INFRASTRUCTURE ONLY): each example built
unchanged with g++ from the reference sources by tests/refsuite/build.py
(oracle/_ref/examples/<name>) and run here; stdout and the exit code go to
tests/golden/reference_examples.json, which tests/test_refsuite_gpu.py
compares the device builds of the same examples with.

Usage: python tests/golden/make_reference_outputs.py
"""
import importlib.util
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
_spec = importlib.util.spec_from_file_location("plx_refsuite_build",
                                               ROOT / "tests" / "refsuite" / "build.py")
refsuite = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(refsuite)


def main() -> int:
    if not refsuite.available():
        print("reference tree not found", file=sys.stderr)
        return 1
    out = {}
    for d in refsuite.EXAMPLES:
        exe = refsuite.build_reference_example(d)
        r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
        out[refsuite.example_name(d)] = {"returncode": r.returncode, "stdout": r.stdout}
        print(f"{d}: rc={r.returncode}, {len(r.stdout.splitlines())} lines")
    path = ROOT / "tests" / "golden" / "reference_examples.json"
    path.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
