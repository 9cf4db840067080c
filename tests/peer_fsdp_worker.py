"""Worker of tests/test_peer_fsdp_multigpu.py (one process per GPU under torchrun, NCCL).

A small bf16 model is trained for three steps with PeerShardedOptimizer (the NVLink kernel of
csrc/peer_optim.cu) and, on the side, with an fp32 AdamW restatement on the NCCL-averaged
gradients of the same inputs. Checks: parameters agree with the restatement, and every rank holds
a bitwise-identical replica after each step."""

import copy
import os
import sys

import torch
import torch.distributed as dist
from torch import nn

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    from tiny_dsv41_b200 import ops
    from tiny_dsv41_b200.parallel.peer_fsdp import PeerShardedOptimizer

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(256, 1000), nn.Tanh(), nn.Linear(1000, 129), nn.Tanh(), nn.Linear(129, 64))
    model = model.to(dev, torch.bfloat16)
    if rank == 1:
        with torch.no_grad():
            for p in model.parameters():
                p.mul_(3.0)  # replicas must start from rank 0's values
    units = [list(model[0].parameters()), list(model[2].parameters()), list(model[4].parameters())]
    lr, wd, b1, b2, eps = 1e-2, 0.1, 0.9, 0.95, 1e-8
    opt = PeerShardedOptimizer(units, algo="adamw", lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd)
    shadow = copy.deepcopy(model)
    master = [p.detach().float().clone() for p in shadow.parameters()]
    m = [torch.zeros_like(x) for x in master]
    v = [torch.zeros_like(x) for x in master]
    for step in range(1, 4):
        gen = torch.Generator(device=dev).manual_seed(1000 * step + rank)
        x = torch.randn(96, 256, device=dev, dtype=torch.bfloat16, generator=gen)
        opt.begin_step()
        model(x).float().square().mean().backward()
        opt.finish_step()
        shadow.zero_grad()
        shadow(x).float().square().mean().backward()
        for i, p in enumerate(shadow.parameters()):
            g = p.grad.float()
            dist.all_reduce(g)
            g /= world
            master[i].mul_(1 - lr * wd)
            m[i].mul_(b1).add_(g, alpha=1 - b1)
            v[i].mul_(b2).addcmul_(g, g, value=1 - b2)
            master[i].addcdiv_(m[i], v[i].sqrt() / (1 - b2 ** step) ** 0.5 + eps, value=-lr / (1 - b1 ** step))
            with torch.no_grad():
                p.copy_(master[i])
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        ref = flat.clone()
        dist.broadcast(ref, 0)  # bf16 broadcast copies the bits
        assert torch.equal(flat, ref), f"replicas differ after step {step}"
    torch.cuda.synchronize()
    ops.check_status("peer_update")
    for p, q in zip(model.parameters(), master):
        torch.testing.assert_close(p.detach().float(), q, rtol=2e-2, atol=2e-3)
    dist.barrier()
    if rank == 0:
        print("PEER_FSDP OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
