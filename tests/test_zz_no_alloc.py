"""plx_compact_noalloc: the compaction entry point that allocates nothing.

Some callers cannot allocate device memory at the moment they compact (a
step loop with a fixed memory budget, a host framework that owns every device
allocation). This entry point keeps its scratch in a static device array
instead of caller-provided or library-allocated scratch. The test calls it
through the C ABI twice in a row (different sizes and data, so the second
call must clear what the first left behind) and compares every output with
the regular plx_compact, bit for bit (compaction is exact integer/byte work).
It creates all of its inputs itself, so it passes alone in a fresh process
as well as after the other tests. This file is collected last.
"""
from ctypes import c_void_p

import numpy as np
import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import Context, _fields, compact

pytestmark = pytest.mark.gpu

LIMIT = 1 << 28


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.1, n).astype(np.float32)
    f = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.int32)
    age = rng.integers(0, 256, n, dtype=np.uint8)
    return [torch.from_numpy(x).cuda() for x in (w, f, age)]


def _run_noalloc(stream, n, w, f, age):
    outs = [torch.zeros_like(w), torch.zeros_like(f), torch.zeros_like(age)]
    perm = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    fields = _fields([(w, outs[0]), (f, outs[1]), (age, outs[2])],
                     [0, 0, _abi.FIELD_INC_SAT_U8])
    rc = _abi.lib().plx_compact_noalloc(c_void_p(stream.cuda_stream), n, _abi.KEEP_ABS_GE,
                                        c_void_p(w.data_ptr()), 0.02, fields, 3,
                                        c_void_p(perm.data_ptr()), c_void_p(count.data_ptr()))
    _abi.check(rc, "plx_compact_noalloc")
    return outs, perm, count


def _run_regular(ctx, n, w, f, age):
    outs = [torch.zeros_like(w), torch.zeros_like(f), torch.zeros_like(age)]
    perm = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    compact(ctx, n, _abi.KEEP_ABS_GE, w, [(w, outs[0]), (f, outs[1]), (age, outs[2])],
            count, threshold=0.02, flags=[0, 0, _abi.FIELD_INC_SAT_U8], perm_out=perm)
    return outs, perm, count


def test_noalloc_compaction_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = Context(0)
    stream = torch.cuda.current_stream()
    # Two calls in a row: the second is smaller and must not see the first
    # call's tile words or count.
    for n, seed in ((3_000_017, 1), (40_961, 2)):
        w, f, age = _inputs(n, seed)
        got = _run_noalloc(stream, n, w, f, age)
        want = _run_regular(ctx, n, w, f, age)
        ctx.sync()
        m = int(want[2].item())
        assert int(got[2].item()) == m
        assert 0 < m < n
        for g, x in zip(got[0], want[0]):
            np.testing.assert_array_equal(g[:m].cpu().numpy(), x[:m].cpu().numpy())
        np.testing.assert_array_equal(got[1][:m].cpu().numpy(), want[1][:m].cpu().numpy())
    ctx.close()


def test_noalloc_rejects_sizes_above_its_limit():
    lib = _abi.lib()
    rc = lib.plx_compact_noalloc(None, LIMIT + 1, _abi.KEEP_FLAGS, c_void_p(16), 0.0, None,
                                 0, None, c_void_p(16))
    assert rc == _abi.PLX_ERR_ARG
    assert b"limit" in lib.plx_last_error()


def test_noalloc_empty_input_counts_zero():
    # n = 0 after a non-empty call: the count must come back 0, as from the
    # regular entry point, not the previous call's count.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = Context(0)
    stream = torch.cuda.current_stream()
    w, f, age = _inputs(10_000, 3)
    _run_noalloc(stream, 10_000, w, f, age)
    empty = [t[:0] for t in (w, f, age)]
    got = _run_noalloc(stream, 0, *empty)
    want = _run_regular(ctx, 0, *empty)
    ctx.sync()
    assert int(got[2].item()) == int(want[2].item()) == 0
    ctx.close()
