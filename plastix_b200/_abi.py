"""ctypes bindings of ``libplastix_b200.so`` (declared in include/plastix_b200.h).

The library is the product: there is no Python or CPU fallback. Loading
fails with an ImportError-style exception when the shared library is missing.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libplastix_b200.so")

PLX_OK = 0
PLX_ERR_ARG = 1
PLX_ERR_CUDA = 2
PLX_ERR_CAPACITY = 3
PLX_ERR_TIMEOUT = 4
PLX_ERR_UNSUPPORTED = 5

APPLY_IDENTITY = 0
APPLY_SIGMOID = 1
APPLY_TANH = 2
APPLY_IPC_ERROR = 3
APPLY_SIGMOID_GRAD = 4
APPLY_TANH_GRAD = 5

UPDATE_GRADIENT = 1
UPDATE_HEBBIAN = 2
UPDATE_HEBBIAN_T = 3

SEQ_ROW_MAX = 256
CHUNK_SOURCES = 16384
MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class PlxError(RuntimeError):
    def __init__(self, code: int, where: str, message: str):
        super().__init__(f"{where} failed with status {code}: {message}")
        self.code = code


class Csr(ctypes.Structure):
    _fields_ = [("row_ptr", c_void_p), ("plan", c_void_p), ("to_id", c_void_p),
                ("n_edges", c_uint64), ("n_rows", c_uint32), ("row_base", c_uint32),
                ("n_wide", c_uint32), ("n_long", c_uint32), ("n_short", c_uint32),
                ("max_row", c_uint32)]


class Chunked(ctypes.Structure):
    _fields_ = [("seg_ptr", c_void_p), ("src", c_void_p), ("perm", c_void_p),
                ("n_rows", c_uint32), ("n_src", c_uint32), ("n_chunks", c_uint32)]


class Sliced(ctypes.Structure):
    _fields_ = [("slice_ptr", c_void_p), ("lane_row", c_void_p), ("lane_len", c_void_p),
                ("perm", c_void_p), ("n_slots", c_uint64), ("n_edges", c_uint64),
                ("n_rows", c_uint32), ("n_slices", c_uint32)]


SLICED_NONE = 0xFFFFFFFF


class Field(ctypes.Structure):
    _fields_ = [("src", c_void_p), ("dst", c_void_p), ("elem_bytes", c_uint32),
                ("flags", c_uint32)]


KEEP_FLAGS = 0
KEEP_NOT_DEAD = 1
KEEP_ABS_GE = 2
FIELD_INC_SAT_U8 = 1
COUNT_UNKNOWN = 0xFFFFFFFF
MAX_FIELDS = 16

# name -> (restype, argtypes)
_SIGNATURES = {
    "plx_version": (c_char_p, []),
    "plx_last_error": (c_char_p, []),
    "plx_ctx_create": (c_int, [c_int, c_void_p, POINTER(c_void_p)]),
    "plx_ctx_destroy": (c_int, [c_void_p]),
    "plx_ctx_set_stream": (c_int, [c_void_p, c_void_p]),
    "plx_ctx_set_timeout_ns": (c_int, [c_void_p, c_uint64]),
    "plx_ctx_num_sms": (c_int, [c_void_p, POINTER(c_int)]),
    "plx_ctx_sync": (c_int, [c_void_p]),
    "plx_csr_row_ptr": (c_int, [c_void_p, c_void_p, c_uint64, c_uint32, c_uint32, c_void_p]),
    "plx_csr_plan_words": (c_uint64, [c_uint64, c_uint32]),
    "plx_csr_plan": (c_int, [c_void_p, c_void_p, c_uint32, c_uint64, c_void_p, c_uint64,
                             c_void_p]),
    "plx_csr_plan_async": (c_int, [c_void_p, c_void_p, c_uint32, c_uint64, c_void_p,
                                   c_uint64, c_void_p]),
    "plx_compact_scratch_bytes": (ctypes.c_size_t, [c_uint64]),
    "plx_compact": (c_int, [c_void_p, c_uint64, c_int, c_void_p, c_float, c_void_p,
                            c_uint32, c_void_p, c_void_p, c_void_p, ctypes.c_size_t]),
    "plx_compact_noalloc": (c_int, [c_void_p, c_uint64, c_int, c_void_p, c_float, c_void_p,
                                    c_uint32, c_void_p, c_void_p]),
    "plx_gather": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_uint32]),
    "plx_radix_sort_scratch_bytes": (ctypes.c_size_t, [c_uint64]),
    "plx_radix_sort_u32": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p,
                                   c_uint32, c_uint32, c_void_p, ctypes.c_size_t]),
    "plx_sweep_forward_rows": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_uint32, c_int, c_void_p, c_void_p,
                                       c_void_p]),
    "plx_sort_tail_scratch_bytes": (ctypes.c_size_t, [c_uint64]),
    "plx_sort_tail_u32": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_uint32, c_uint32, c_void_p, ctypes.c_size_t]),
    "plx_transpose_scratch_bytes": (ctypes.c_size_t, [c_uint64]),
    "plx_transpose": (c_int, [c_void_p, c_uint64, c_void_p, c_uint32, c_uint32, c_int, c_void_p,
                              c_void_p, c_void_p, c_void_p, ctypes.c_size_t]),
    "plx_ipc_value_update": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_float,
                                     c_void_p, c_int]),
    "plx_mse_sigmoid_grad": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p]),
    "plx_chunked_max_padded": (c_uint64, [c_uint64, c_uint32, c_uint32]),
    "plx_chunked_scratch_bytes": (ctypes.c_size_t, [c_uint64, c_uint32, c_uint32]),
    "plx_chunked_build": (c_int, [c_void_p, c_uint64, c_void_p, c_uint32, c_uint32, c_void_p,
                                  c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p,
                                  ctypes.c_size_t]),
    "plx_chunked_gather": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p]),
    "plx_chunked_fold": (c_int, [c_void_p, POINTER(Chunked), c_void_p, c_void_p, c_int,
                                 c_void_p, c_void_p, c_void_p]),
    "plx_chunked_update": (c_int, [c_void_p, POINTER(Chunked), c_void_p, c_void_p, c_void_p,
                                   c_int, c_float]),
    "plx_chunked_fold_ipc_value": (c_int, [c_void_p, POINTER(Chunked), c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_float, c_void_p, c_void_p]),
    "plx_sweep_forward_hebbian_gather": (c_int, [c_void_p, POINTER(Csr), c_void_p, c_void_p,
                                                 c_void_p, c_uint32, c_void_p, c_void_p,
                                                 c_void_p, c_void_p, c_float, c_float,
                                                 c_void_p, c_void_p, c_uint32, c_uint32,
                                                 c_uint32]),
    "plx_peer_alloc": (c_int, [c_void_p, ctypes.c_size_t, POINTER(c_void_p), c_void_p]),
    "plx_peer_free": (c_int, [c_void_p, c_void_p]),
    "plx_peer_open": (c_int, [c_void_p, c_void_p, POINTER(c_void_p)]),
    "plx_peer_close": (c_int, [c_void_p, c_void_p]),
    "plx_peer_barrier": (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_uint64]),
    "plx_copy_device": (c_int, [c_void_p, c_void_p, c_void_p, ctypes.c_size_t]),
    "plx_recompute_levels_scratch_bytes": (ctypes.c_size_t, [c_uint64, c_uint64]),
    "plx_recompute_levels": (c_int, [c_void_p, c_uint32, c_uint32, c_uint64, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t]),
    "plx_src_levels": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_uint32, c_void_p]),
    "plx_sort_unique_u64_scratch_bytes": (ctypes.c_size_t, [c_uint64]),
    "plx_sort_unique_u64": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    ctypes.c_size_t]),
    "plx_swifttd_scratch_bytes": (c_uint64, [c_uint64, c_uint32]),
    "plx_swifttd_step": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_uint32,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_uint64]),
    "plx_swifttd_reduce": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_uint32,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_uint64]),
    "plx_swifttd_apply": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_uint32,
                                  c_void_p, c_void_p, c_uint64]),
    "plx_regrow": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_uint64,
                           c_uint64]),
    "plx_sweep_forward": (c_int, [c_void_p, POINTER(Csr), c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_uint32, c_int, c_void_p, c_void_p, c_void_p]),
    "plx_sweep_forward_hebbian": (c_int, [c_void_p, POINTER(Csr), c_void_p, c_void_p,
                                          c_void_p, c_uint32, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_float, c_float, c_void_p]),
    "plx_sweep_update": (c_int, [c_void_p, POINTER(Csr), c_void_p, c_void_p, c_void_p,
                                 c_uint32, c_void_p, c_int, c_float, c_void_p, c_void_p]),
    "plx_sliced_n_slices": (c_uint32, [c_uint32]),
    "plx_sliced_plan_scratch_bytes": (ctypes.c_size_t, [c_uint32]),
    "plx_sliced_plan": (c_int, [c_void_p, c_void_p, c_uint32, c_uint64, POINTER(Sliced),
                                c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t]),
    "plx_sliced_perm": (c_int, [c_void_p, POINTER(Sliced), c_void_p, c_void_p]),
    "plx_sliced_pack": (c_int, [c_void_p, POINTER(Sliced), c_void_p, c_void_p, c_uint32]),
    "plx_sliced_unpack": (c_int, [c_void_p, POINTER(Sliced), c_void_p, c_void_p, c_uint32]),
    "plx_sweep_forward_hebbian_sliced": (c_int, [c_void_p, POINTER(Sliced), c_void_p, c_void_p,
                                                 c_void_p, c_uint32, c_void_p, c_void_p,
                                                 c_float, c_float, c_void_p, c_void_p,
                                                 c_uint32, c_uint32, c_uint32]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m plastix_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(code: int, where: str) -> None:
    if code != PLX_OK:
        msg = lib().plx_last_error().decode(errors="replace")
        raise PlxError(code, where, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
