"""Tensor-parallel decoding on 2, 4 and 8 GPUs (one process per GPU; the
residual stream exchanged through peer memory or NCCL) against the oracle;
each world size is skipped when the box has fewer GPUs."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("case,exchange", [("small", "nccl"), ("small", "peer"), ("full", "peer"),
                                           ("switch", "peer")])
def test_tensor_parallel(case, exchange, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), "--case", case, "--exchange", exchange]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_rank_stops(world):
    """A rank that stops calling between steps: the other ranks' next step
    ends with VOX_ERR_DEVICE_TIMEOUT (bounded peer waits), not a hang."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), "--case", "leave", "--exchange", "peer"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
