"""Context-parallel attention kernels (csrc/attention.cu: attn_fwd_cp / attn_bwd_cp /
attn_cp_finalize) against a plain fp32 PyTorch restatement of causal GQA attention.

On one GPU the CP ranks are emulated one after another: each "rank" gets its own chunk of the
queries and the list of every chunk's K / V buffers (local memory standing in for the peer
mappings), writes its own outbox, and each owner then sums its slot of all outboxes. No launch
waits on another. The multi-GPU test runs the same path over NVLink through the autograd
wrapper in tiny_dsv41_b200.parallel.cp_attention.
"""

import os
import subprocess
import sys

import pytest
import torch

from tests.test_attention_gpu import _inputs, _rel, reference
from tiny_dsv41_b200 import ops

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _chunks(t, n):
    return [c.contiguous() for c in t.chunk(n, dim=1)]


@pytest.mark.parametrize("batch,seq,heads,kv_heads,cp", [(1, 512, 4, 2, 2), (2, 768, 8, 2, 3), (1, 1024, 4, 1, 4)])
def test_cp_forward_backward_matches_full_sequence(batch, seq, heads, kv_heads, cp):
    q, k, v = _inputs(batch, seq, heads, kv_heads, seed=3)
    chunk = seq // cp
    qs, ks, vs = _chunks(q, cp), _chunks(k, cp), _chunks(v, cp)
    kp = [t.data_ptr() for t in ks]
    vp = [t.data_ptr() for t in vs]
    outs, lses = [], []
    for r in range(cp):
        out, lse = ops.ext().attn_fwd_cp(qs[r], kp, vp, chunk, r * chunk, kv_heads)
        outs.append(out)
        lses.append(lse)
    ops.check_status("attn_fwd_cp")
    out = torch.cat(outs, dim=1)
    ref_out, ref_lse = reference(q, k, v)
    assert _rel(out, ref_out) < 1e-2
    assert torch.allclose(torch.cat(lses, dim=2), ref_lse, atol=2e-3, rtol=1e-3)
    # the non-CP kernel on the full sequence gives the same forward
    full, _ = ops.ext().attn_fwd(q, k, v)
    assert _rel(out, full) < 1e-3

    g = torch.Generator(device="cuda").manual_seed(9)
    dout = torch.randn(q.shape, device="cuda", generator=g).to(torch.bfloat16)
    douts = _chunks(dout, cp)
    boxes = [torch.empty(cp, 2, batch, chunk, kv_heads, 128, device="cuda") for _ in range(cp)]
    dqs = [ops.ext().attn_bwd_cp(douts[r], qs[r], kp, vp, outs[r], lses[r], chunk, r * chunk, kv_heads, boxes[r])
           for r in range(cp)]
    table = torch.tensor([b.data_ptr() for b in boxes], dtype=torch.int64, device="cuda")
    dks, dvs = zip(*(ops.ext().attn_cp_finalize(table, c, batch, chunk, kv_heads) for c in range(cp)))
    ops.check_status("attn_bwd_cp")
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ref, _ = reference(qr, kr, vr)
    ref.backward(dout.float())
    assert _rel(torch.cat(dqs, dim=1), qr.grad) < 2e-2
    assert _rel(torch.cat(dks, dim=1), kr.grad) < 2e-2
    assert _rel(torch.cat(dvs, dim=1), vr.grad) < 2e-2


@pytest.mark.multigpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_cp_attention_2gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29641",
           os.path.join(ROOT, "tests", "cp_attention_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "CP_ATTENTION OK" in proc.stdout
