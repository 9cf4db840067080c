"""Pieces shared by the model families."""

from __future__ import annotations

import torch
from torch import nn

from .. import ops


class LMHead(nn.Linear):
    """``nn.Linear`` LM head whose forward can also return the fused cross-entropy sum or
    selected-token log-probabilities.

    Going through ``forward`` matters under FSDP2: the (sharded) weight is only gathered inside
    the module's forward, so the loss kernels must run there rather than on ``self.weight``
    from an enclosing module.
    """

    def __init__(self, hidden_size: int, vocab_size: int) -> None:
        super().__init__(hidden_size, vocab_size, bias=False)

    def forward(self, hidden: torch.Tensor, targets: torch.Tensor | None = None, *, mode: str = "logits",
                temperature: float = 1.0) -> torch.Tensor:
        if mode == "logits":
            return ops.linear(hidden, self.weight)
        if mode == "ce_sum":
            return ops.linear_cross_entropy(hidden.reshape(-1, hidden.shape[-1]), self.weight, targets.reshape(-1))
        if mode == "logprob":
            logits = ops.linear(hidden, self.weight).float()
            return ops.token_log_probs(logits, targets, temperature)
        raise ValueError(f"unknown LM head mode {mode!r}")


__all__ = ["LMHead"]


class Linear(nn.Linear):
    """``nn.Linear`` (same parameters and state-dict keys) whose forward runs the tcgen05 GEMM."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = ops.linear(x, self.weight)
        return out if self.bias is None else out + self.bias.to(out.dtype)


def fusable(*modules: nn.Module) -> bool:
    """True when the modules are plain projections whose weights may be concatenated into one GEMM
    (an injected LoRA adapter disables the fusion for its module)."""
    return all(type(m) is Linear and m.bias is None for m in modules)


__all__ += ["Linear", "fusable"]
