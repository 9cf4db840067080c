"""FSDP2 wrapping for both model families.

Layout (the reference wraps the same units: ``dsv41_train/models/dsv4/parallel.py`` and
``dsv41_train/models/qwen/parallel.py``):

* dense parameters shard over the whole world (data and context-parallel ranks alike: a CP
  rank's gradient is its token shard's contribution, so the world-wide reduce-scatter is the
  full gradient);
* routed experts are placed by expert parallelism; when the world is larger than the EP size
  their replicas shard over the ``expert_fsdp`` mesh, otherwise FSDP ignores them;
* fp32 islands (mHC mixing, attention sinks) are separate fp32 units, so bf16 mixed precision
  never casts them;
* Engram tables (row-sharded or host-offloaded) stay outside FSDP;
* each unit prefetches only itself in backward, so FSDP collectives never interleave with the
  EP exchange of a neighbouring layer in a rank-dependent order.
"""

from __future__ import annotations

import torch
from torch import nn


def expert_parameters(model: nn.Module) -> list[nn.Parameter]:
    from ..models.dsv4.moe import RoutedExperts
    from ..models.qwen.model import Qwen3MoeExperts

    return [p for m in model.modules() if isinstance(m, (RoutedExperts, Qwen3MoeExperts)) for p in m.parameters()]


def _fp32_islands(layer: nn.Module) -> list[nn.Module]:
    from ..models.dsv4.attention import AttentionSinks
    from ..models.dsv4.mhc import HyperConnection

    return [m for m in layer.modules() if isinstance(m, (HyperConnection, AttentionSinks))]


def apply_fsdp(model: nn.Module, meshes, *, param_dtype=torch.bfloat16, reduce_dtype=torch.float32,
               reshard_after_forward: bool = True) -> None:
    from torch.distributed.fsdp import FSDPModule, MixedPrecisionPolicy, fully_shard

    from ..models.dsv4.moe import RoutedExperts
    from ..models.qwen.model import Qwen3MoeExperts

    mesh = meshes.fsdp if meshes.cp is None else meshes.dense_world
    policy = MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=reduce_dtype)
    fp32_policy = MixedPrecisionPolicy(param_dtype=torch.float32, reduce_dtype=torch.float32)
    opts = {"mesh": mesh, "mp_policy": policy, "reshard_after_forward": reshard_after_forward}
    experts_sharded = meshes.ep is not None and meshes.expert_fsdp is not None and meshes.expert_fsdp.size() > 1
    ignored: set = set()
    for m in model.modules():
        if isinstance(m, (RoutedExperts, Qwen3MoeExperts)):
            if experts_sharded:
                fully_shard(m, mesh=meshes.expert_fsdp, mp_policy=policy, reshard_after_forward=reshard_after_forward)
            elif meshes.ep is not None:
                ignored.update(m.parameters())
    engram = getattr(getattr(model, "model", None), "engram_tables", None)
    if engram is not None:
        ignored.update(engram.parameters())
    inner = model.model
    embed = getattr(inner, "embed_tokens", None) or getattr(inner, "embedding", None)
    fully_shard(embed, **opts)
    for layer in inner.layers:
        for island in _fp32_islands(layer):
            fully_shard(island, mesh=mesh, mp_policy=fp32_policy, reshard_after_forward=reshard_after_forward)
        fully_shard(layer, ignored_params=ignored, **opts)
    fully_shard(model.lm_head, **opts)
    # the root keeps its parameters gathered between forward and backward: its output is a
    # dataclass, which no pre-backward hook can attach to
    fully_shard(model, mesh=mesh, mp_policy=policy, ignored_params=ignored)
    for module in model.modules():
        if isinstance(module, FSDPModule):
            module.set_modules_to_backward_prefetch([module])




def scale_expert_grads(model: nn.Module, ep_size: int) -> None:
    """Expert gradients arrive summed over the EP group's per-rank losses while FSDP averages the
    dense ones over the world; dividing them by the EP size puts both on the same scale (the
    expert-FSDP reduce-scatter, when experts are replicated, already divides by world / ep)."""
    if ep_size <= 1:
        return
    for p in expert_parameters(model):
        if p.grad is not None:
            p.grad.mul_(1.0 / ep_size)


@torch.no_grad()
def clip_grad_norm_(parameters, max_norm: float) -> torch.Tensor:
    """Global L2 norm over sharded (DTensor) and rank-local gradients, then in-place clipping.

    Every rank holds a distinct piece of the gradient (FSDP shards, or this EP rank's experts),
    so the squared norms of the local pieces sum to the global one with one all-reduce."""
    import torch.distributed as dist

    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return torch.zeros(())
    local = [g.to_local() if hasattr(g, "to_local") else g for g in grads]
    device = local[0].device
    sq = torch.zeros((), device=device, dtype=torch.float32)
    for g in local:
        sq += g.float().square().sum()
    if dist.is_initialized():
        dist.all_reduce(sq)
    norm = sq.sqrt()
    if not bool(torch.isfinite(norm)):
        raise FloatingPointError("non-finite gradient norm; optimizer step not applied")
    coef = min(1.0, max_norm / (float(norm) + 1e-6))
    if coef < 1.0:
        for g in local:
            g.mul_(coef)
    return norm


__all__ = ["apply_fsdp", "clip_grad_norm_", "expert_parameters", "scale_expert_grads"]
