"""RMSNorm (fp32 statistics, activation-dtype rounding before the weight multiply).

Reference semantics: ``dsv41_train/models/qwen/model.py:45-57`` and
``dsv41_train/models/dsv4/attention/module.py:20-30``.
"""

from __future__ import annotations

import torch

from ._ext import ext, on_gpu


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    normalized = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + eps)
    return normalized.to(x.dtype) * weight


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, rstd = ext().rmsnorm_fwd(x2, weight.contiguous(), float(eps))
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        need_dw = ctx.needs_input_grad[1]
        dx, dw = ext().rmsnorm_bwd(dy.reshape(x2.shape).contiguous(), x2, weight.contiguous(), rstd, need_dw)
        return dx.view(ctx.shape), (dw.to(weight.dtype) if need_dw else None), None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if on_gpu(x) and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
        return _RMSNorm.apply(x, weight, eps)
    return rms_norm_reference(x, weight, eps)
