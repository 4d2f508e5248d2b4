"""Real multi-GPU runs (one process per GPU over CUDA IPC and NVLink) of the
fused path against the reference's PyTorch + NCCL path; see
tests/mgpu_worker.py for the cases.  Skipped with fewer than two GPUs."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_multi_gpu_world():
    n = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "60", "900", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(HERE, "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=os.path.dirname(HERE))
    print(r.stdout[-8000:])
    if r.returncode != 0:
        print(r.stderr[-8000:])
    assert r.returncode == 0
    assert f"MULTI-GPU RESULT world={n}: PASS" in r.stdout
