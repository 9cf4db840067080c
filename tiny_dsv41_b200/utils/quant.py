"""FP8 / FP4 (OCP MX) codecs for the released DeepSeek-V4.1 checkpoint layout.

* FP8 E4M3 weights with one E8M0 (power-of-two) scale per 32x32 block, or per 32 columns of a row.
* FP4 E2M1 weights packed two per byte (low nibble first) with one E8M0 scale per 32 values
  along the input dimension - the MXFP4 layout that tcgen05 ``kind::mxf4`` consumes directly.

The E2M1 code points are the OCP Microscaling spec's: 0, 0.5, 1, 1.5, 2, 3, 4, 6 and negatives.
"""

from __future__ import annotations

import torch

E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


@torch.no_grad()
def dequantize_fp8_blocks(weight: torch.Tensor, scale: torch.Tensor, *, dtype=torch.bfloat16) -> torch.Tensor:
    if weight.ndim != 2 or scale.ndim != 2:
        raise ValueError("FP8 weight and scale must both be matrices")
    out_f, in_f = weight.shape
    ob, ib = scale.shape
    if out_f != ob * 32 or in_f != ib * 32:
        raise ValueError(f"FP8 shape mismatch: weight={tuple(weight.shape)}, scale={tuple(scale.shape)}")
    blocks = weight.view(ob, 32, ib, 32).float()
    return (blocks * scale.float()[:, None, :, None]).reshape(weight.shape).to(dtype)


@torch.no_grad()
def dequantize_fp8_rows(weight: torch.Tensor, scale: torch.Tensor, *, dtype=torch.bfloat16) -> torch.Tensor:
    if weight.ndim != 2 or scale.ndim != 2:
        raise ValueError("FP8 weight and scale must both be matrices")
    rows, feats = weight.shape
    if scale.shape[0] != rows or feats != scale.shape[1] * 32:
        raise ValueError(f"row-scaled FP8 shape mismatch: weight={tuple(weight.shape)}, scale={tuple(scale.shape)}")
    return (weight.view(rows, scale.shape[1], 32).float() * scale.float().unsqueeze(-1)).flatten(1).to(dtype)


@torch.no_grad()
def dequantize_fp4_rows(packed: torch.Tensor, scale: torch.Tensor, *, dtype=torch.bfloat16) -> torch.Tensor:
    if packed.dtype not in (torch.int8, torch.uint8) or packed.ndim != 2 or scale.ndim != 2:
        raise ValueError("FP4 weight must be an int8 matrix with a matrix of scales")
    out_f, packed_f = packed.shape
    if scale.shape[0] != out_f or packed_f * 2 != scale.shape[1] * 32:
        raise ValueError(f"FP4 shape mismatch: weight={tuple(packed.shape)}, scale={tuple(scale.shape)}")
    table = torch.tensor(E2M1_VALUES, device=packed.device, dtype=torch.float32)
    raw = packed.view(torch.uint8)
    values = torch.stack((table[(raw & 0x0F).long()], table[(raw >> 4).long()]), dim=-1).flatten(1)
    return (values.view(out_f, scale.shape[1], 32) * scale.float().unsqueeze(-1)).flatten(1).to(dtype)


def _e8m0(exponent: torch.Tensor) -> torch.Tensor:
    """Power-of-two scales 2**exponent as an E8M0 tensor (or fp32 if the dtype is missing)."""
    value = torch.pow(2.0, exponent.float())
    return value.to(torch.float8_e8m0fnu) if hasattr(torch, "float8_e8m0fnu") else value


@torch.no_grad()
def quantize_fp4_rows(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """MXFP4 encoding: per 32 values a power-of-two scale with amax/scale <= 6, nearest E2M1 code."""
    rows, feats = weight.shape
    if feats % 32:
        raise ValueError("FP4 rows need a multiple of 32 values")
    blocks = weight.float().view(rows, feats // 32, 32)
    amax = blocks.abs().amax(-1).clamp_min(1e-30)
    exponent = torch.ceil(torch.log2(amax / 6.0))
    scale = torch.pow(2.0, exponent)
    scaled = blocks / scale.unsqueeze(-1)
    table = torch.tensor(E2M1_VALUES[:8], device=weight.device)
    codes = (scaled.abs().unsqueeze(-1) - table).abs().argmin(-1)
    codes = codes + 8 * (scaled < 0).long()
    codes = codes.view(rows, feats).to(torch.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    return packed, _e8m0(exponent)


@torch.no_grad()
def quantize_fp8_blocks(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    out_f, in_f = weight.shape
    blocks = weight.float().view(out_f // 32, 32, in_f // 32, 32)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-30)
    exponent = torch.ceil(torch.log2(amax / 448.0))
    scale = torch.pow(2.0, exponent)
    q = (blocks / scale[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(out_f, in_f)
    return q, _e8m0(exponent)


@torch.no_grad()
def quantize_fp8_rows(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    rows, feats = weight.shape
    blocks = weight.float().view(rows, feats // 32, 32)
    exponent = torch.ceil(torch.log2(blocks.abs().amax(-1).clamp_min(1e-30) / 448.0))
    q = (blocks / torch.pow(2.0, exponent).unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(rows, feats)
    return q, _e8m0(exponent)


__all__ = ["E2M1_VALUES", "dequantize_fp4_rows", "dequantize_fp8_blocks", "dequantize_fp8_rows", "quantize_fp4_rows",
           "quantize_fp8_blocks", "quantize_fp8_rows"]
