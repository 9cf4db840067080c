"""Context parallelism and NCCL-baseline expert parallelism on 2 gloo CPU ranks vs one process."""

import torch
import torch.distributed as dist

from dist_utils import run_gloo


def _cp_worker(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from tiny_dsv41_b200.parallel.cp import ContextParallel

    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("cp",))
    cp = ContextParallel(mesh)
    torch.manual_seed(0)
    full = torch.randn(2, 8, 3, requires_grad=True)
    local = cp.shard(full.detach()).requires_grad_()
    gathered = cp.gather(local, dim=1)
    assert torch.equal(gathered, full.detach())
    weights = torch.arange(8.0).view(1, 8, 1).expand(2, 8, 3)
    (gathered * weights).sum().backward()
    # every rank contributes the same upstream gradient, so the local grad is world x the slice
    expected = (weights * world).chunk(world, dim=1)[rank]
    assert torch.allclose(local.grad, expected)
    x = cp.shard(full.detach()).requires_grad_()
    halo = cp.left_halo(x, 2, dim=1)
    if rank == 0:
        assert halo.shape[1] == 4
    else:
        assert torch.equal(halo[:, :2], full.detach()[:, rank * 4 - 2: rank * 4])
    halo.sum().backward()
    grad = torch.ones_like(x)
    if rank < world - 1:
        grad[:, -2:] += 1
    assert torch.equal(x.grad, grad)
    loss = cp.mean_loss(torch.tensor(3.0 + rank), torch.tensor(2 + rank))
    assert abs(loss.item() - (3 + 4) / (2 + 3)) < 1e-6


def test_context_parallel_gloo():
    run_gloo(_cp_worker, 2)


def _ep_worker(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from tiny_dsv41_b200.ops import gemm as G
    from tiny_dsv41_b200.ops import moe as M
    from tiny_dsv41_b200.parallel.dispatch import AllToAllTokenDispatcher, TokenDispatcher

    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("ep",))
    e, k, h, inter, t = 8, 2, 16, 8, 12
    gen = torch.Generator().manual_seed(0)
    w1 = torch.randn(e, 2 * inter, h, generator=gen)
    w2 = torch.randn(e, h, inter, generator=gen)
    gen.manual_seed(10 + rank)
    x = torch.randn(t, h, generator=gen)
    probs = torch.softmax(torch.randn(t, e, generator=gen), -1)
    w, ids = probs.topk(k, -1)
    ids = ids.to(torch.int32)
    local_e = e // world
    sl = slice(rank * local_e, (rank + 1) * local_e)

    def run(disp, w1p, w2p, xp, wp):
        batch = disp.dispatch(xp, ids, wp)
        gu = G.grouped_linear(batch.rows, w1p, batch.offsets, batch.sizes)
        y = G.grouped_linear(M.swiglu(gu), w2p, batch.offsets, batch.sizes)
        return disp.combine(y, batch, weighted=True)

    dist_disp = AllToAllTokenDispatcher(mesh)
    dist_disp.expert_range(e)
    xa, wa = x.clone().requires_grad_(), w.clone().requires_grad_()
    w1a, w2a = w1[sl].clone().requires_grad_(), w2[sl].clone().requires_grad_()
    out = run(dist_disp, w1a, w2a, xa, wa)
    out.sum().backward()
    local = TokenDispatcher()
    local.expert_range(e)
    xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()
    w1r, w2r = w1.clone().requires_grad_(), w2.clone().requires_grad_()
    ref = run(local, w1r, w2r, xr, wr)
    ref.sum().backward()
    assert torch.allclose(out, ref, atol=1e-4)
    assert torch.allclose(xa.grad, xr.grad, atol=1e-4)
    assert torch.allclose(wa.grad, wr.grad, atol=1e-4)
    g1 = w1r.grad.clone()
    dist.all_reduce(g1)
    assert torch.allclose(w1a.grad, g1[sl], atol=1e-3)


def test_expert_parallel_nccl_baseline_on_gloo():
    run_gloo(_ep_worker, 2)


def test_build_routing_masks_and_segments():
    from tiny_dsv41_b200.ops.moe import build_routing

    ids = torch.tensor([[0, 2], [2, -1], [1, 0]], dtype=torch.int32)
    r = build_routing(ids, 3, block=4)
    assert r.offsets.tolist() == [0, 4, 8]
    assert r.rows.tolist() == [4, 4, 4]
    assert r.route_rows[1, 1].item() == -1
    assert int(r.total) == 12
    src = r.src.tolist()
    assert src[0] == 0 and src[1] == 2 and src[4] == 2 and src[8] == 0 and src[9] == 1
