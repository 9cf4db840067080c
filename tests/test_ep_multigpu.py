"""Expert parallelism over NVLink on 2+ GPUs (torchrun child processes, NVLS off)."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_dispatch_combine_parity_2gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29631",
           os.path.join(ROOT, "tests", "ep_parity_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "EP_PARITY OK" in proc.stdout


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_guard_rows_stay_intact_2gpu():
    """Debug mode TDSV_EP_CANARY=1: guard rows after the peer-written slabs are checked after every
    dispatch and combine of the parity run."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_NCCL_ASYNC_ERROR_HANDLING="1", TDSV_EP_CANARY="1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29637",
           os.path.join(ROOT, "tests", "ep_parity_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "EP_PARITY OK" in proc.stdout
