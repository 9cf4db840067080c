"""Fused gradient reduce-scatter + AdamW + parameter gather over NVLink on 2 GPUs (torchrun child
processes, NVLS off)."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_sharded_adamw_2gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29641",
           os.path.join(ROOT, "tests", "peer_fsdp_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    where = proc.stderr.find("Traceback")
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[max(where, 0):][:4000]
    assert "PEER_FSDP OK" in proc.stdout
