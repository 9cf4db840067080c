"""Frozen MXFP4 expert weights: kept packed, expanded to bf16 only while a GEMM needs them.

``dequantize_fp4`` runs the sm_100a kernel on CUDA tensors and the plain PyTorch restatement on
CPU. ``fp4_grouped_linear`` is the grouped GEMM against a frozen packed weight: the forward
expands the weight, multiplies and drops the expanded copy; the backward (input gradient only -
the weight is frozen) expands it again instead of keeping it alive between the passes.
"""

from __future__ import annotations

import torch

from ..utils.quant import E2M1_VALUES
from ._ext import ext, on_gpu
from .gemm import grouped_linear, grouped_linear_reference


def dequantize_fp4(packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """uint8 codes [..., C/2] (low nibble first) and uint8 E8M0 scales [..., C/32] -> bf16 [..., C]."""
    if on_gpu(packed):
        return ext().fp4_dequant(packed.contiguous(), scale.contiguous())
    table = torch.tensor(E2M1_VALUES, dtype=torch.float32)
    raw = packed.to(torch.uint8)
    values = torch.stack((table[(raw & 0x0F).long()], table[(raw >> 4).long()]), dim=-1).flatten(-2)
    scales = torch.pow(2.0, scale.float() - 127.0)
    shape = values.shape
    blocks = values.reshape(*shape[:-1], shape[-1] // 32, 32) * scales.unsqueeze(-1)
    return blocks.reshape(shape).to(torch.bfloat16)


class _FrozenFP4GroupedLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, packed, scale, offsets, rows, out_features):
        weight = dequantize_fp4(packed, scale).view(packed.shape[0], out_features, -1)
        ctx.save_for_backward(packed, scale, offsets, rows)
        ctx.out_features = out_features
        return grouped_linear(x, weight, offsets, rows)

    @staticmethod
    def backward(ctx, dy):
        packed, scale, offsets, rows = ctx.saved_tensors
        weight = dequantize_fp4(packed, scale).view(packed.shape[0], ctx.out_features, -1)
        dy = dy.contiguous()
        # dx = dy @ W per expert segment
        if on_gpu(dy):
            dx = torch.empty(dy.shape[0], weight.shape[2], dtype=torch.bfloat16, device=dy.device)
            ext().grouped_gemm_m(dy, weight, offsets, rows, dx, True, dy.shape[0])
        else:
            dx = grouped_linear_reference(dy, weight.transpose(1, 2), offsets, rows)
        return dx, None, None, None, None, None


def fp4_grouped_linear(x, packed, scale, offsets, rows, out_features: int) -> torch.Tensor:
    """Rows of ``x`` in expert segments times the frozen packed weight ``[G, out_features, in]``."""
    return _FrozenFP4GroupedLinear.apply(x, packed, scale, offsets, rows, out_features)


__all__ = ["dequantize_fp4", "fp4_grouped_linear"]
