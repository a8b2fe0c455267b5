"""Failure detection without a GPU fault: every wait in a kernel is bounded
and ends in a status the host reads. Here the cross-GPU barrier waits for a
peer flag that nothing ever sets (both "ranks'" flag arrays live on this one
GPU and only rank 0 runs): the kernel gives up after the context's timeout,
records TIMEOUT, and the context stays usable."""
import ctypes
import time

import pytest
import torch

from plastix_b200 import _abi
from plastix_b200.runtime import Context

pytestmark = pytest.mark.gpu


def test_peer_barrier_times_out_and_reports(ctx):
    lib = _abi.lib()
    c = Context(0)
    c.set_timeout_ns(200_000_000)  # 0.2 s
    flags = [torch.zeros(2, dtype=torch.int64, device="cuda") for _ in range(2)]
    arr = (ctypes.c_void_p * 2)(*[f.data_ptr() for f in flags])
    t0 = time.time()
    _abi.call("plx_peer_barrier", c.handle, arr, 2, 0, 1)
    with pytest.raises(_abi.PlxError) as e:
        c.sync()
    assert e.value.code == _abi.PLX_ERR_TIMEOUT
    assert time.time() - t0 < 10
    # rank 0 published its epoch into "rank 1"'s array; nothing else changed
    assert int(flags[1][0].item()) == 1 and int(flags[0][1].item()) == 0
    # the status was read and cleared: the context keeps working
    x = torch.ones(1000, device="cuda")
    assert float(x.sum().item()) == 1000.0
    c.sync()
    # a barrier whose peer flag is already set passes at once
    flags[0][1].fill_(5)
    _abi.call("plx_peer_barrier", c.handle, arr, 2, 0, 2)
    c.sync()
    c.close()
