"""Several GPUs (2, 4 and 8 ranks, each where the machine has that many):
the sharded multilayer iPC network (unit-range shards, NCCL all-gathers of
f(x) and eps) equals the same network on one GPU bit for bit, on every rank;
the fused sweep + peer-memory hand-off (stores over NVLink, bounded barrier)
equals the plain sweep + NCCL all-gather bit for bit; and a recurrent chain of
hand-offs (each sweep reads the previous epoch's gathered buffer, no host
synchronisation between steps) equals the unsharded layer on one GPU."""
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


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ipc_and_peer_handoff(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), str(WORKER)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
