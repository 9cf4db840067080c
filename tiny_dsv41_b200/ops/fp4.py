"""Frozen MXFP4 expert weights, kept packed and multiplied packed.

``dequantize_fp4`` runs the sm_100a kernel on CUDA tensors and the plain PyTorch restatement on
CPU. ``fp4_grouped_linear`` is the grouped GEMM against a frozen packed weight: on CUDA both the
forward and the input gradient (the weight is frozen) run the tcgen05 grouped GEMM whose weight
producers convert E2M1 codes with their E8M0 scales to bf16 in shared memory, so the weight is
never expanded in global memory; on CPU the weight is dequantised and multiplied in fp32.
"""

from __future__ import annotations

import torch

from ..utils.quant import E2M1_VALUES
from ._ext import ext, on_gpu
from .gemm import grouped_linear_reference


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
    """Forward and input gradient read the packed weight directly (``fp4_grouped_gemm``): the codes
    and scales cross HBM at 4.25 bits per value and no bf16 copy of the weight is ever written."""

    @staticmethod
    def forward(ctx, x, packed, scale, offsets, rows, out_features):
        out = torch.empty(x.shape[0], out_features, dtype=torch.bfloat16, device=x.device)
        ext().fp4_grouped_gemm(x, packed, scale, offsets, rows, out, False, x.shape[0])
        ctx.save_for_backward(packed, scale, offsets, rows)
        return out

    @staticmethod
    def backward(ctx, dy):
        packed, scale, offsets, rows = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.empty(dy.shape[0], packed.shape[2] * 2, dtype=torch.bfloat16, device=dy.device)
        ext().fp4_grouped_gemm(dy, packed, scale, offsets, rows, dx, True, dy.shape[0])
        return dx, None, None, None, None, None


def _fp4_reference(x, packed, scale, offsets, rows, out_features):
    weight = dequantize_fp4(packed, scale).view(packed.shape[0], out_features, -1)
    return grouped_linear_reference(x, weight, offsets, rows)


def fp4_grouped_linear(x, packed, scale, offsets, rows, out_features: int) -> torch.Tensor:
    """Rows of ``x`` in expert segments times the frozen packed weight ``[G, out_features, in]``
    (codes ``[G, out_features, in / 2]``, scales ``[G, out_features, in / 32]``)."""
    in_features = packed.shape[2] * 2
    if on_gpu(x) and x.dtype == torch.bfloat16 and in_features % 64 == 0 and out_features % 64 == 0:
        return _FrozenFP4GroupedLinear.apply(x.contiguous(), packed.contiguous(), scale.contiguous(), offsets, rows,
                                             out_features)
    return _fp4_reference(x, packed, scale, offsets, rows, out_features)


__all__ = ["dequantize_fp4", "fp4_grouped_linear"]
