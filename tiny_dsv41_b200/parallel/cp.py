"""Context parallelism over a packed token stream.

The batch is flattened into one stream and split into equal contiguous shards per CP rank
(``dsv41_train/cp.py:119-270`` has the same contract). Provided here:

* :class:`ContextParallel` - shard / autograd all-gather (backward = reduce-scatter) /
  sliding-window left halo from the previous rank (backward returns the halo gradient) /
  autograd sum / CP-correct mean loss.
* :class:`ModelContext` - per-token positions that restart at every packed sequence,
  sliding-window key indices relative to the halo-extended local shard and the window mask.
* :func:`pack_sequences`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING

import torch
import torch.distributed as dist
import torch.nn.functional as F

if TYPE_CHECKING:
    from torch.distributed.device_mesh import DeviceMesh


def _reduce_scatter_sum(grad: torch.Tensor, group, size: int) -> torch.Tensor:
    """Sum of the `size` equal chunks (dim 0) of `grad` over the group, chunk `rank` kept."""
    if dist.get_backend(group) == "nccl":
        out = grad.new_empty((grad.shape[0] // size, *grad.shape[1:]))
        dist.reduce_scatter_tensor(out, grad.contiguous(), group=group)
        return out
    exchanged = torch.empty_like(grad)
    dist.all_to_all_single(exchanged, grad.contiguous(), group=group)
    return torch.stack(exchanged.chunk(size, dim=0)).sum(0)


class _AllGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, dim, group, size):
        ctx.meta = (dim, group, size)
        moved = tensor.movedim(dim, 0).contiguous()
        out = moved.new_empty((moved.shape[0] * size, *moved.shape[1:]))
        dist.all_gather_into_tensor(out, moved, group=group)
        return out.movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, grad):
        dim, group, size = ctx.meta
        local = _reduce_scatter_sum(grad.movedim(dim, 0).contiguous(), group, size)
        return local.movedim(0, dim).contiguous(), None, None, None


def _shift(tensor: torch.Tensor, *, to_next: bool, group) -> torch.Tensor:
    """Send `tensor` to the next (or previous) rank of the ring and receive the opposite one."""
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    peer_send = (rank + 1) % size if to_next else (rank - 1) % size
    peer_recv = (rank - 1) % size if to_next else (rank + 1) % size
    received = torch.empty_like(tensor)
    global_send = dist.get_global_rank(group, peer_send)
    global_recv = dist.get_global_rank(group, peer_recv)
    ops = [dist.P2POp(dist.isend, tensor.contiguous(), global_send, group),
           dist.P2POp(dist.irecv, received, global_recv, group)]
    for work in dist.batch_isend_irecv(ops):
        work.wait()
    return received


class _LeftHalo(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, length, dim, group):
        rank = dist.get_rank(group)
        ctx.meta = (rank, dist.get_world_size(group), length, dim, group)
        tail = tensor.narrow(dim, tensor.shape[dim] - length, length).movedim(dim, 0).contiguous()
        prefix = _shift(tail, to_next=True, group=group).movedim(0, dim)
        return tensor if rank == 0 else torch.cat((prefix, tensor), dim=dim)

    @staticmethod
    def backward(ctx, grad):
        rank, size, length, dim, group = ctx.meta
        if rank == 0:
            shape = list(grad.shape)
            shape[dim] = length
            prefix_grad, local = grad.new_zeros(shape), grad
        else:
            prefix_grad = grad.narrow(dim, 0, length)
            local = grad.narrow(dim, length, grad.shape[dim] - length)
        received = _shift(prefix_grad.movedim(dim, 0).contiguous(), to_next=False, group=group).movedim(0, dim)
        result = local.clone()
        if rank < size - 1:
            result.narrow(dim, result.shape[dim] - length, length).add_(received)
        return result, None, None, None


class ContextParallel:
    """Token sharding and the collectives sequence modules need under CP."""

    def __init__(self, mesh: "DeviceMesh | None" = None, *, fused_attention: bool = True) -> None:
        self.mesh = mesh
        self.size = 1 if mesh is None else mesh.size()
        self.rank = 0 if mesh is None else mesh.get_local_rank()
        self.group = None if mesh is None else mesh.get_group()
        # causal attention with the K/V exchange inside the kernels (parallel.cp_attention) for
        # inputs with default positions and no padding mask; set per forward by the model
        self.fused_attention = fused_attention
        self.plain_causal = False
        self._fused = None

    def fused(self, num_layers: int):
        """The model's fused CP attention (created on first use; CUDA only)."""
        if self._fused is None:
            from .cp_attention import FusedCPAttention

            self._fused = FusedCPAttention(self.group, num_layers)
        return self._fused

    @property
    def enabled(self) -> bool:
        return self.size > 1

    def shard(self, tensor: torch.Tensor, dim: int = 1) -> torch.Tensor:
        if not self.enabled:
            return tensor
        if tensor.shape[dim] % self.size:
            raise ValueError(f"dimension {dim} ({tensor.shape[dim]}) must divide CP size ({self.size})")
        return tensor.chunk(self.size, dim=dim)[self.rank].contiguous()

    def gather(self, tensor: torch.Tensor, dim: int = 1) -> torch.Tensor:
        if not self.enabled:
            return tensor
        if tensor.requires_grad:
            return _AllGather.apply(tensor.contiguous(), dim, self.group, self.size)
        moved = tensor.movedim(dim, 0).contiguous()
        out = moved.new_empty((moved.shape[0] * self.size, *moved.shape[1:]))
        dist.all_gather_into_tensor(out, moved, group=self.group)
        return out.movedim(0, dim).contiguous()

    def left_halo(self, tensor: torch.Tensor, length: int, dim: int = 1) -> torch.Tensor:
        if not self.enabled or length == 0:
            return tensor
        if not 0 <= length <= tensor.shape[dim]:
            raise ValueError(f"halo length ({length}) must be in [0, {tensor.shape[dim]}]")
        return _LeftHalo.apply(tensor.contiguous(), length, dim, self.group)

    def sum(self, tensor: torch.Tensor, *, autograd: bool = False) -> torch.Tensor:
        if not self.enabled:
            return tensor
        if autograd:
            import torch.distributed.nn.functional as dist_nn

            return dist_nn.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self.group)
        result = tensor.clone()
        dist.all_reduce(result, op=dist.ReduceOp.SUM, group=self.group)
        return result

    def mean_loss(self, local_sum: torch.Tensor, local_count: torch.Tensor) -> torch.Tensor:
        """Global CP mean value; the backward path is scaled so FSDP gradient averaging stays exact."""
        if not self.enabled:
            return local_sum / local_count.clamp_min(1)
        total = self.sum(local_sum.detach())
        count = self.sum(local_count.detach()).clamp_min(1)
        backward_loss = local_sum * (self.size / count)
        return backward_loss + (total / count - backward_loss.detach())


@dataclass(frozen=True)
class ModelContext:
    parallel: ContextParallel
    input_ids: torch.Tensor
    positions: torch.Tensor
    token_mask: torch.Tensor
    sequence_ids: torch.Tensor
    attention_indices: torch.Tensor
    attention_mask: torch.Tensor
    attention_halo_length: int

    @classmethod
    def build(cls, parallel: ContextParallel, input_ids: torch.Tensor, token_mask: torch.Tensor,
              sequence_ids: torch.Tensor, window: int) -> "ModelContext":
        length = input_ids.shape[1]
        index = torch.arange(length, device=input_ids.device).expand_as(input_ids)
        previous = F.pad(sequence_ids[:, :-1], (1, 0), value=-1)
        starts = token_mask & (sequence_ids != previous)
        last_start = torch.where(starts, index, torch.zeros_like(index)).cummax(-1).values
        positions = (index - last_start).masked_fill(~token_mask, 0)
        local_index = parallel.shard(index)
        keys = local_index.unsqueeze(-1) - torch.arange(window - 1, -1, -1, device=input_ids.device)
        in_range = keys >= 0
        keys = keys.clamp_min(0)
        key_seq = sequence_ids.gather(1, keys.flatten(1)).view_as(keys)
        key_live = token_mask.gather(1, keys.flatten(1)).view_as(keys)
        local_ids, local_pos, local_mask, local_seq = map(parallel.shard, (input_ids, positions, token_mask,
                                                                            sequence_ids))
        local_len = local_ids.shape[1]
        halo = window - 1 if parallel.enabled and window - 1 <= local_len else 0
        if halo:
            prefix = 0 if parallel.rank == 0 else halo
            attention_indices = keys - parallel.rank * local_len + prefix
        else:
            attention_indices = keys
        mask = in_range & key_live & local_mask.unsqueeze(-1) & (local_seq.unsqueeze(-1) == key_seq)
        return cls(parallel, local_ids, local_pos, local_mask, local_seq, attention_indices, mask.unsqueeze(1), halo)

    def gather(self, tensor: torch.Tensor, dim: int = 1) -> torch.Tensor:
        return self.parallel.gather(tensor, dim)

    def gather_attention(self, tensor: torch.Tensor, dim: int = 1) -> torch.Tensor:
        if self.attention_halo_length:
            return self.parallel.left_halo(tensor, self.attention_halo_length, dim)
        return self.parallel.gather(tensor, dim)


def pack_sequences(input_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Flatten [B, L] into one stream and return (packed ids [1, B*L], sequence ids [1, B*L])."""
    batch, length = input_ids.shape
    sequence_ids = torch.arange(batch, device=input_ids.device).repeat_interleave(length)
    return input_ids.reshape(1, -1), sequence_ids.reshape(1, -1)


__all__ = ["ContextParallel", "ModelContext", "pack_sequences"]
