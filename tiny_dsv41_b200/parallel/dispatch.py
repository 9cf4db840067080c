"""Expert-parallel token dispatch.

Common contract (used by the Qwen and DSV4 expert modules)::

    dispatcher.expert_range(num_experts) -> (start, stop)         # experts owned by this rank
    batch = dispatcher.dispatch(x [T, H], ids [T, k] int, weights [T, k] fp32)
    # batch.rows:   expert-major rows [R, H], each local expert a 128-row aligned segment
    # batch.offsets / batch.sizes: int32 [E_local] device tensors for the grouped GEMMs
    # batch.row_weights: fp32 [R] route weight of every row (0 on padding rows)
    out = dispatcher.combine(y_rows [R, H], batch, weighted=True)  # [T, H]

* :class:`TokenDispatcher` - single rank (EP=1): gather into expert-major order, fp32 top-k sum
  in router-slot order.
* :class:`AllToAllTokenDispatcher` - EP over NCCL ``all_to_all_single`` with host-synchronised
  split sizes: the behaviour of ``dsv41_train/dispatch.py:46-146`` and the baseline the fused
  NVLink dispatcher (``parallel/nvlink_ep.py``) is measured against.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
import torch.distributed.nn.functional as dist_nn

from .. import ops
from ..ops import moe as moe_ops


@dataclass
class DispatchBatch:
    rows: torch.Tensor
    offsets: torch.Tensor
    sizes: torch.Tensor
    row_weights: torch.Tensor | None
    state: dict[str, Any] = field(default_factory=dict)
    total: torch.Tensor | None = None  # int32 device scalar: rows in use


def _row_weights(routing: moe_ops.Routing, weights: torch.Tensor) -> torch.Tensor:
    """fp32 [R_cap] weight of each expert-major row (0 for padding)."""
    out = torch.zeros(routing.capacity, dtype=torch.float32, device=weights.device)
    out.index_put_((routing.route_rows.reshape(-1).long(),), weights.reshape(-1).float())
    return out


class _ScatterWeights(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weights, route_rows, capacity):
        ctx.save_for_backward(route_rows)
        out = torch.zeros(capacity, dtype=torch.float32, device=weights.device)
        out[route_rows.reshape(-1).long()] = weights.reshape(-1).float()
        return out

    @staticmethod
    def backward(ctx, grad):
        (route_rows,) = ctx.saved_tensors
        return grad[route_rows.long()], None, None


class TokenDispatcher:
    """All experts local (EP=1)."""

    def __init__(self) -> None:
        self.num_experts: int | None = None
        self.size = 1
        self.rank = 0

    def end_step(self) -> None:
        """Called once per training step after its backward; the local dispatcher keeps no state."""

    def abort_step(self) -> None:
        """Forget the exchanges counted for a step that did not run (a failed graph capture)."""

    def expert_range(self, num_experts: int) -> tuple[int, int]:
        if num_experts < 1:
            raise ValueError("num_experts must be positive")
        self.num_experts = num_experts
        return 0, num_experts

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> DispatchBatch:
        if self.num_experts is None:
            raise RuntimeError("attach the dispatcher to an expert module before use")
        routing = moe_ops.build_routing(ids, self.num_experts)
        rows = moe_ops.gather(x, routing)
        return DispatchBatch(rows, routing.offsets, routing.rows, None,
                             {"routing": routing, "weights": weights}, routing.total)

    def row_weights(self, batch: DispatchBatch) -> torch.Tensor:
        routing = batch.state["routing"]
        return _ScatterWeights.apply(batch.state["weights"], routing.route_rows, routing.capacity)

    def combine(self, y: torch.Tensor, batch: DispatchBatch, *, weighted: bool = True) -> torch.Tensor:
        routing = batch.state["routing"]
        return moe_ops.combine(y, routing, batch.state["weights"] if weighted else None)


class AllToAllTokenDispatcher(TokenDispatcher):
    """EP over NCCL all-to-all (one token copy per route, host-synchronised splits)."""

    def __init__(self, mesh) -> None:
        super().__init__()
        if mesh.ndim != 1:
            raise ValueError("the EP mesh must be one-dimensional")
        self.mesh = mesh
        self.size = mesh.size()
        self.rank = mesh.get_local_rank()
        self.group = mesh.get_group()

    def expert_range(self, num_experts: int) -> tuple[int, int]:
        if num_experts % self.size:
            raise ValueError(f"num_experts ({num_experts}) must divide EP size ({self.size})")
        self.num_experts = num_experts
        local = num_experts // self.size
        return self.rank * local, (self.rank + 1) * local

    def _exchange(self, tensor, out_splits, in_splits, autograd):
        out = tensor.new_empty((sum(out_splits), *tensor.shape[1:]))
        if autograd:
            return dist_nn.all_to_all_single(out, tensor, output_split_sizes=out_splits,
                                             input_split_sizes=in_splits, group=self.group)
        dist.all_to_all_single(out, tensor, output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)
        return out

    def dispatch(self, x, ids, weights):
        if self.num_experts is None:
            raise RuntimeError("attach the dispatcher to an expert module before use")
        tokens, k = ids.shape
        local = self.num_experts // self.size
        flat = ids.reshape(-1).long()
        owners = torch.div(flat, local, rounding_mode="floor")
        order = torch.argsort(owners, stable=True)
        send = torch.bincount(owners, minlength=self.size)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        send_splits, recv_splits = send.tolist(), recv.tolist()
        token_of_route = torch.div(order, k, rounding_mode="floor")
        sent_rows = x[token_of_route]
        recv_ids = self._exchange((flat[order] - owners[order] * local).to(torch.int32).contiguous(),
                                  recv_splits, send_splits, False)
        recv_rows = self._exchange(sent_rows.contiguous(), recv_splits, send_splits, True)
        recv_weights = self._exchange(weights.reshape(-1)[order].float().contiguous(), recv_splits,
                                      send_splits, True)
        routing = moe_ops.build_routing(recv_ids.view(-1, 1), local)
        rows = moe_ops.gather(recv_rows, routing)
        state = {"routing": routing, "weights": recv_weights.view(-1, 1), "order": order,
                 "send_splits": send_splits, "recv_splits": recv_splits, "tokens": tokens, "k": k}
        return DispatchBatch(rows, routing.offsets, routing.rows, None, state, routing.total)

    def combine(self, y, batch, *, weighted: bool = True):
        s = batch.state
        per_route = moe_ops.combine(y, s["routing"], s["weights"] if weighted else None)
        returned = self._exchange(per_route.contiguous(), s["send_splits"], s["recv_splits"], True)
        restored = torch.empty_like(returned)
        restored = restored.index_copy(0, s["order"], returned)
        return restored.view(s["tokens"], s["k"], -1).float().sum(1).to(y.dtype)


__all__ = ["AllToAllTokenDispatcher", "DispatchBatch", "TokenDispatcher"]
