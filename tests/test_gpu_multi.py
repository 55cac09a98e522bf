"""Multi-GPU (one process per GPU, the library's NCCL layer): the data-parallel
model step equals the single-GPU full-batch step, the batch-sharded Scan-A /
convnd backward reductions equal the full-batch gradients, the output gather
assembles every rank's y (tests/mp_model_dp.py); skipped with fewer than 2 GPUs."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_data_parallel_model_two_gpus(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(ROOT, "tests", "mp_model_dp.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=240,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0", KMB_DIST_CHECK="1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
