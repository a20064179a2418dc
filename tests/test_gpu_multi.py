"""Fused row-sharded projection + argmax + peer-memory exchange on every
visible GPU (2..8); skipped on a single-GPU machine.  Each rank is its own
process (torchrun) on its own GPU, as in serving."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_exchange_all_visible_gpus(cuda):
    n = min(cuda.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs at least two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "multigpu_exchange_check.py")]
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
