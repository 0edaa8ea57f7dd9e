"""GPU, two or more devices: heads sharded over two ranks (one process per GPU, NCCL), no collective on the
compute path; the outputs gathered to rank 0 equal a single-GPU run of all heads bit for bit.

Skipped on a machine with one GPU. The ranks run as torchrun children (tests/multigpu_worker.py) with a
short process-group timeout and an outer time limit, so a lost rank ends the test with an error.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_heads_gathered_to_rank0_equal_single_gpu(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(HERE, "multigpu_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert p.returncode == 0 and "MULTIGPU_OK" in p.stdout, (p.stdout[-3000:], p.stderr[-3000:])
