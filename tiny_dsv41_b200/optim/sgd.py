"""SGD applied inside the backward pass (``dsv41_train/optim.py:13-137`` semantics).

A post-accumulate-grad hook updates each (local shard of a) parameter as soon as its gradient
is ready, optionally through an fp32 master, scales expert gradients by a divisor, and raises a
device-side non-finite flag instead of synchronising; the caller all-reduces the flag (MIN of
"finite") and aborts the run if any rank saw a non-finite gradient.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..ops import ext
from ..runtime import local_tensor


@dataclass
class SGDInBackward:
    lr: float
    divisors: dict[int, float]
    masters: dict[int, torch.Tensor]
    flag: torch.Tensor
    handles: list = field(default_factory=list)

    def finite(self) -> bool:
        return int(self.flag.item()) == 0

    def reset(self) -> None:
        self.flag.zero_()

    def remove(self) -> None:
        for handle in self.handles:
            handle.remove()
        self.handles.clear()


def install_sgd_in_backward(params, lr: float, *, expert_divisor: float = 1.0, expert_params=(),
                            fp32_master: bool = False, grad_scale: float = 1.0) -> SGDInBackward:
    params = [p for p in params if p.requires_grad]
    expert_ids = {id(p) for p in expert_params}
    device = params[0].device if params else torch.device("cpu")
    state = SGDInBackward(lr, {}, {}, torch.zeros(1, dtype=torch.int32, device=device))
    for p in params:
        state.divisors[id(p)] = expert_divisor if id(p) in expert_ids else 1.0
        if fp32_master:
            state.masters[id(p)] = local_tensor(p.data).detach().float().clone()

    @torch.no_grad()
    def hook(p: torch.Tensor) -> None:
        grad = local_tensor(p.grad)
        data = local_tensor(p.data)
        scale = grad_scale / state.divisors[id(p)]
        master = state.masters.get(id(p))
        if grad.is_sparse:  # row-sparse embedding gradients (Engram tables): update only the touched rows
            g = grad.coalesce()
            rows, values = g.indices()[0], g.values().float() * scale
            bad = (~torch.isfinite(values)).any().to(state.flag.dtype).reshape(1)
            state.flag.copy_(torch.maximum(state.flag, bad.to(state.flag.device)))
            target = master if master is not None else data
            target.index_add_(0, rows.to(target.device), (-lr * values).to(device=target.device, dtype=target.dtype))
            if master is not None:
                data[rows] = master[rows].to(data.dtype)
        elif data.is_cuda:
            target = master if master is not None else data
            out = data if (master is not None and data.dtype == torch.bfloat16) else None
            ext().sgd_step(target, grad.contiguous(), out, lr, scale, state.flag)
            if master is not None and out is None:
                data.copy_(master)
        else:
            g = grad.float() * scale
            if not torch.isfinite(g).all():
                state.flag.fill_(1)
            target = master if master is not None else data
            target.sub_(g.to(target.dtype), alpha=lr)
            if master is not None:
                data.copy_(master)
        p.grad = None

    for p in params:
        state.handles.append(p.register_post_accumulate_grad_hook(hook))
    return state


__all__ = ["SGDInBackward", "install_sgd_in_backward"]
