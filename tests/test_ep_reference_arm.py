"""bench_ep.py's reference expert arms (the reference's DeepSeek-V4 RoutedExperts on its own
dispatcher, and the Qwen per-expert loop) run one forward + backward on two CPU gloo ranks when the
unmodified reference is installed in baseline/_ref."""

import os
import subprocess
import sys

import pytest

from ref_oracle import reference_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not reference_available(), reason="the reference package is not installed in baseline/_ref")
@pytest.mark.timeout(600)
def test_reference_expert_arms_run_on_gloo():
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", "29741",
                          os.path.join(ROOT, "tests", "ep_reference_arm_worker.py")],
                         cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, OMP_NUM_THREADS="2"))
    assert out.returncode == 0, out.stderr[-3000:]
    for rank in (0, 1):
        for arm in ("dsv4", "qwen"):
            assert f"rank {rank} arm {arm} ok" in out.stdout, out.stdout[-2000:]
