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


def test_peer_slice_past_the_peer_buffers_is_rejected_before_any_device_work():
    # The fused sweep stores row r to peer_out[p][peer_offset + r]: a slice
    # that does not fit the peer buffers must fail as an argument error
    # before the context (here a dummy, never dereferenced) or any device
    # memory is touched.
    import ctypes

    lib = _abi.lib()
    fake_ctx = ctypes.c_void_p(0x1000)
    csr = _abi.Csr(row_ptr=0x2000, plan=0x3000, to_id=None, n_edges=0, n_rows=100,
                   row_base=0, n_wide=0, n_long=0, n_short=100, max_row=0)
    peers = (ctypes.c_void_p * 2)(0x4000, 0x5000)
    args = [fake_ctx, ctypes.byref(csr), None, None, None, 0, None, None, None, None,
            0.9, 1e-3, ctypes.c_void_p(0x6000), peers, 2]
    assert lib.plx_sweep_forward_hebbian_gather(*args, 150, 200) == _abi.PLX_ERR_ARG
    assert b"exceeds the peer buffers" in lib.plx_last_error()
    assert lib.plx_sweep_forward_hebbian_gather(*args, 0, 99) == _abi.PLX_ERR_ARG
