"""Worker for the multi-GPU expert-parallel parity test (launched by torchrun, one rank per GPU).

Every rank routes its own tokens through experts sharded over the EP group with the NVLink
dispatcher and compares output, input gradient, route-weight gradient and local expert weight
gradients with a single-rank computation over the full (replicated) expert set.
"""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from tiny_dsv41_b200 import ops  # noqa: E402
from tiny_dsv41_b200.ops import gemm as G  # noqa: E402
from tiny_dsv41_b200.ops import moe as M  # noqa: E402
from tiny_dsv41_b200.parallel.dispatch import AllToAllTokenDispatcher, TokenDispatcher  # noqa: E402
from tiny_dsv41_b200.parallel.nvlink_ep import NVLinkTokenDispatcher  # noqa: E402


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def experts_forward(dispatcher, x, ids, w, w1, w2, weighted_in_swiglu):
    batch = dispatcher.dispatch(x, ids, w)
    gu = G.grouped_linear(batch.rows, w1, batch.offsets, batch.sizes)
    if weighted_in_swiglu:
        act = M.swiglu(gu, dispatcher.row_weights(batch), total=batch.total)
        y = G.grouped_linear(act, w2, batch.offsets, batch.sizes)
        return dispatcher.combine(y, batch, weighted=False)
    act = M.swiglu(gu, total=batch.total)
    y = G.grouped_linear(act, w2, batch.offsets, batch.sizes)
    return dispatcher.combine(y, batch, weighted=True)


def main():
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    rank, world = dist.get_rank(), dist.get_world_size()
    from torch.distributed.device_mesh import init_device_mesh

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("ep",))
    dev = torch.device("cuda", local_rank)
    t, h, e, k, inter = 300, 256, 8 * world, 4, 128
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    w1_full = torch.randn(e, 2 * inter, h, device=dev, generator=gen, dtype=torch.bfloat16) * 0.05
    w2_full = torch.randn(e, h, inter, device=dev, generator=gen, dtype=torch.bfloat16) * 0.05
    gen.manual_seed(100 + rank)
    x = torch.randn(t, h, device=dev, generator=gen, dtype=torch.bfloat16)
    logits = torch.randn(t, e, device=dev, generator=gen)
    w = torch.softmax(logits, -1).topk(k, -1).values
    ids = torch.softmax(logits, -1).topk(k, -1).indices.to(torch.int32)
    dout = torch.randn(t, h, device=dev, generator=gen, dtype=torch.bfloat16)
    e_local = e // world
    sl = slice(rank * e_local, (rank + 1) * e_local)
    failures = []
    from torch.utils.checkpoint import checkpoint

    from tiny_dsv41_b200.parallel import replay

    cases = [("nvlink", NVLinkTokenDispatcher, False), ("nccl", AllToAllTokenDispatcher, False),
             ("nvlink-ckpt", NVLinkTokenDispatcher, True)]
    for name, cls, ckpt in cases:
        for weighted_in_swiglu in (False, True):
            for trial in range(2):  # second trial exercises the epoch / free-flag reuse path
                disp = cls(mesh)
                disp.expert_range(e)
                xa = x.clone().requires_grad_()
                wa = w.clone().requires_grad_()
                w1 = w1_full[sl].clone().requires_grad_()
                w2 = w2_full[sl].clone().requires_grad_()
                if ckpt:  # the recompute replays the recorded exchanges instead of repeating them
                    out = checkpoint(experts_forward, disp, xa, ids, wa, w1, w2, weighted_in_swiglu,
                                     use_reentrant=False, context_fn=replay.checkpoint_contexts)
                    out.backward(dout)
                    ws = disp._ws
                    if (ws.recv_epoch, ws.ret_epoch) != (2, 2):
                        failures.append((name, "exchanges", ws.recv_epoch, ws.ret_epoch))
                else:
                    out = experts_forward(disp, xa, ids, wa, w1, w2, weighted_in_swiglu)
                    out.backward(dout)
                local = TokenDispatcher()
                local.expert_range(e)
                xr = x.clone().requires_grad_()
                wr = w.clone().requires_grad_()
                w1r = w1_full.clone().requires_grad_()
                w2r = w2_full.clone().requires_grad_()
                ref = experts_forward(local, xr, ids, wr, w1r, w2r, weighted_in_swiglu)
                ref.backward(dout)
                g1 = w1r.grad.float().clone()
                g2 = w2r.grad.float().clone()
                dist.all_reduce(g1)
                dist.all_reduce(g2)
                checks = {"out": rel(out, ref), "dx": rel(xa.grad, xr.grad), "dw": rel(wa.grad, wr.grad),
                          "dw1": rel(w1.grad, g1[sl]), "dw2": rel(w2.grad, g2[sl])}
                bad = {key: v for key, v in checks.items() if not v < 2e-2}
                if bad:
                    failures.append((name, weighted_in_swiglu, trial, bad))
    code = ops.ext().read_status()
    if code:
        failures.append(("status", code))
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        print("EP_PARITY", "FAIL" if failures else "OK", failures, flush=True)
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
