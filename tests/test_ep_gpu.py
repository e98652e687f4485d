"""Expert-parallel decode on two GPUs (tests/ep_gpu_worker.py under torch.distributed.run): every rank's tokens get
the single-device block's bits. Needs two GPUs; skipped on one."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_give_the_single_device_bits():
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ep_gpu_worker.py")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}", worker]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ep bits: same" in r.stdout
