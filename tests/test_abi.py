"""The C ABI library: it loads, exports every function include/plastix_b200.h
declares, and reports errors as status codes (no GPU needed)."""
import re
from pathlib import Path

from plastix_b200 import _abi

HEADER = Path(__file__).resolve().parents[1] / "include" / "plastix_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(plx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = _abi.lib()
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_header():
    assert set(declared_functions()) <= set(_abi.exported_symbols())


def test_version_matches_reference():
    # reference src/plastix.cpp:5 / tests/test_plastix.cpp:8
    assert _abi.lib().plx_version() == b"0.1.0"


def test_null_arguments_are_rejected_without_touching_a_device():
    lib = _abi.lib()
    assert lib.plx_ctx_create(0, None, None) == _abi.PLX_ERR_ARG
    assert b"out" in lib.plx_last_error()
    assert lib.plx_ctx_sync(None) == _abi.PLX_ERR_ARG
    assert lib.plx_sweep_forward(None, None, None, None, None, None, 0, 0, None, None,
                                 None) == _abi.PLX_ERR_ARG


def test_plan_size_formula():
    f = _abi.lib().plx_csr_plan_words
    assert f(0, 0) >= 5
    assert f(64 << 20, 1 << 20) >= (64 << 20) // 256
