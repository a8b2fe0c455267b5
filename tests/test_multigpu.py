"""Several GPUs (runs when the machine has at least two): the sharded
multilayer iPC network (unit-range shards, NCCL all-gathers of f(x) and eps)
equals the same network on one GPU bit for bit, on every rank; and the fused
sweep + peer-memory hand-off (stores over NVLink, bounded barrier) equals the
plain sweep + NCCL all-gather bit for bit."""
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
WORKER = Path(__file__).resolve().parent / "mgpu_worker.py"


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_sharded_ipc_and_peer_handoff_on_two_gpus():
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(_port()), str(WORKER)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
