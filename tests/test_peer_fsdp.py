"""Dense-parameter sync with a sharded optimizer (parallel/peer_fsdp.py): pool layout, the gloo
restatement against torch.optim on averaged gradients, and the fused NVLink kernel on one GPU
against the same fp32 restatement (the multi-GPU run is tests/test_peer_fsdp_multigpu.py)."""

import copy

import pytest
import torch
from torch import nn

from tests.dist_utils import run_gloo
from tiny_dsv41_b200.parallel.peer_fsdp import PeerShardedOptimizer, plan_units


def test_plan_units_alignment_and_cover():
    sizes = [[3, 17, 64], [1], [4096 * 7 + 5, 9]]
    for world in (1, 2, 3, 8):
        layout, total = plan_units(sizes, world)
        cursor = 0
        for (offsets, start, shard), unit in zip(layout, sizes):
            assert start == cursor and start % 8 == 0 and shard % 8 == 0
            assert all(o % 8 == 0 for o in offsets)
            end = offsets[-1] + unit[-1]
            assert end <= start + shard * world  # the shards cover every parameter of the unit
            for a, b, n in zip(offsets, offsets[1:], unit):
                assert b - a >= n
            cursor = start + shard * world
        assert total == cursor


def _model(seed):
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(12, 20), nn.Tanh(), nn.Linear(20, 7), nn.Tanh(), nn.Linear(7, 3))


def _units(model):
    return [list(model[0].parameters()), list(model[2].parameters()), list(model[4].parameters())]


def _reference_params(algo, steps, world, lr, wd):
    """torch.optim on the world-averaged gradient, single process."""
    model = _model(0)
    if algo == "adamw":
        opt = torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd)
    else:
        opt = torch.optim.SGD(model.parameters(), lr=lr)
    for step in range(steps):
        opt.zero_grad()
        for rank in range(world):
            gen = torch.Generator().manual_seed(100 * step + rank)
            x = torch.randn(5, 12, generator=gen)
            (model(x).square().mean() / world).backward()
        opt.step()
    return [p.detach().clone() for p in model.parameters()]


def _gloo_worker(rank, world, algo, steps, lr, wd):
    import torch.distributed as dist

    model = _model(0)
    if rank == 1:  # a different start on rank 1: the optimizer must broadcast rank 0's replica
        with torch.no_grad():
            for p in model.parameters():
                p.add_(1.0)
    opt = PeerShardedOptimizer(_units(model), algo=algo, lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd)
    for step in range(steps):
        opt.begin_step()
        gen = torch.Generator().manual_seed(100 * step + rank)
        x = torch.randn(5, 12, generator=gen)
        model(x).square().mean().backward()
        opt.finish_step()
    expected = _reference_params(algo, steps, world, lr, wd)
    for p, q in zip(model.parameters(), expected):
        torch.testing.assert_close(p.detach(), q, rtol=1e-5, atol=1e-6)
    # every rank holds the same replica
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    other = flat.clone()
    dist.broadcast(other, 0)
    torch.testing.assert_close(flat, other, rtol=0, atol=0)


@pytest.mark.parametrize("algo", ["adamw", "sgd"])
def test_peer_sharded_optimizer_gloo_matches_torch(algo):
    run_gloo(_gloo_worker, 2, algo, 3, 1e-2, 0.1 if algo == "adamw" else 0.0)


def test_unused_parameter_gets_zero_gradient():
    model = _model(0)
    extra = nn.Linear(3, 3)
    opt = PeerShardedOptimizer(_units(model) + [list(extra.parameters())], algo="sgd", lr=0.1)
    before = [p.detach().clone() for p in extra.parameters()]
    opt.begin_step()
    model(torch.randn(4, 12)).sum().backward()
    opt.finish_step()
    for p, q in zip(extra.parameters(), before):
        torch.testing.assert_close(p.detach(), q)  # zero gradient under SGD: unchanged


@pytest.mark.gpu
@pytest.mark.parametrize("moments", [torch.float32, torch.bfloat16])
def test_peer_update_kernel_single_gpu_matches_fp32(moments):
    """world = 1 on one GPU: the fused kernel (peer tables hold the local pools) against an fp32
    AdamW restatement on the same bf16 gradients."""
    dev = torch.device("cuda", 0)
    model = _model(0).to(dev, torch.bfloat16)
    ref_master = [p.detach().float().clone() for p in model.parameters()]
    ref_m = [torch.zeros_like(p) for p in ref_master]
    ref_v = [torch.zeros_like(p) for p in ref_master]
    lr, wd, b1, b2, eps = 1e-2, 0.1, 0.9, 0.95, 1e-8
    opt = PeerShardedOptimizer(_units(model), algo="adamw", lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd,
                               moment_dtype=moments)
    shadow = copy.deepcopy(model)
    for step in range(1, 4):
        x = torch.randn(64, 12, device=dev, dtype=torch.bfloat16)
        opt.begin_step()
        model(x).float().square().mean().backward()
        opt.finish_step()
        # the same gradient on the shadow copy (bf16 weights equal to the pre-update replica)
        shadow.zero_grad()
        shadow(x).float().square().mean().backward()
        for i, p in enumerate(shadow.parameters()):
            g = p.grad.float()
            ref_master[i].mul_(1 - lr * wd)
            ref_m[i].mul_(b1).add_(g, alpha=1 - b1)
            ref_v[i].mul_(b2).addcmul_(g, g, value=1 - b2)
            if moments == torch.bfloat16:
                ref_m[i] = ref_m[i].bfloat16().float()
                ref_v[i] = ref_v[i].bfloat16().float()
            denom = ref_v[i].sqrt() / (1 - b2 ** step) ** 0.5 + eps
            ref_master[i].addcdiv_(ref_m[i], denom, value=-lr / (1 - b1 ** step))
            with torch.no_grad():
                p.copy_(ref_master[i])
    torch.cuda.synchronize()
    for p, q in zip(model.parameters(), ref_master):
        torch.testing.assert_close(p.detach().float(), q, rtol=2e-2, atol=2e-3)
    from tiny_dsv41_b200 import ops

    ops.check_status("peer_update")
