"""Worker for the multi-GPU fused context-parallel attention test (torchrun, one rank per GPU).

Each rank holds one contiguous chunk of a causal sequence. Three layers of attention run through
the fused path (K / V of the other ranks read over NVLink inside the kernels, dK / dV partials
summed by their owner) for two steps, with the second step's forward under activation
checkpointing (record + replay), and every output and gradient is compared with a full-sequence
fp32 computation that every rank does on its own.
"""

import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from tiny_dsv41_b200 import ops  # noqa: E402
from tiny_dsv41_b200.parallel import replay  # noqa: E402
from tiny_dsv41_b200.parallel.cp_attention import FusedCPAttention  # noqa: E402


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def reference(q, k, v):
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    groups = qf.shape[1] // kf.shape[1]
    kf, vf = kf.repeat_interleave(groups, dim=1), vf.repeat_interleave(groups, dim=1)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(q.shape[-1])
    length = q.shape[1]
    s = s.masked_fill(~torch.ones(length, length, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return (torch.softmax(s, dim=-1) @ vf).transpose(1, 2)


def main():
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    rank, world = dist.get_rank(), dist.get_world_size()
    batch, seq, heads, kv_heads, layers = 2, 1024, 8, 2, 3
    chunk = seq // world
    fused = FusedCPAttention(dist.group.WORLD, layers)
    worst = 0.0
    for step in range(2):
        g = torch.Generator(device="cuda").manual_seed(100 + step)  # same full tensors on every rank
        for layer in range(layers):
            q = torch.randn(batch, seq, heads, 128, device="cuda", generator=g).to(torch.bfloat16)
            k = torch.randn(batch, seq, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
            v = torch.randn(batch, seq, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
            dout = torch.randn(batch, seq, heads, 128, device="cuda", generator=g).to(torch.bfloat16)
            sl = slice(rank * chunk, (rank + 1) * chunk)
            ql, kl, vl = (t[:, sl].contiguous().requires_grad_(True) for t in (q, k, v))
            if step == 0:
                out = fused(ql, kl, vl, layer)
            else:  # first forward under "record", then the recompute under "replay" builds the graph
                record, replay_ctx = replay.checkpoint_contexts()
                with record, torch.no_grad():
                    fused(ql.detach(), kl.detach(), vl.detach(), layer)
                with replay_ctx:
                    out = fused(ql, kl, vl, layer)
            out.backward(dout[:, sl])
            qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
            ref = reference(qr, kr, vr)
            ref.backward(dout.float())
            errs = [rel(out, ref[:, sl]), rel(ql.grad, qr.grad[:, sl]), rel(kl.grad, kr.grad[:, sl]),
                    rel(vl.grad, vr.grad[:, sl])]
            worst = max(worst, *errs)
            assert max(errs) < 2e-2, (rank, step, layer, errs)
    ops.check_status("fused CP attention")
    dist.barrier()
    if rank == 0:
        print(f"CP_ATTENTION OK worst rel {worst:.2e}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
