"""Cache fake quantization with a straight-through gradient (DeepSeek-V4 scoring under the
rollout engine's quantized KV cache; reference
``dsv41_train/rl/_native_runtime/c3868011979ca/dsv41_train/models/dsv4/quantization.py``).

``quantize_activation(x, kind)`` returns the values an FP8 / FP4 cache would hand back, in x's dtype,
with the identity as its gradient. Kinds (blocks run along the last dimension; a last dimension
that is not a multiple of the block leaves x unchanged):

* ``"fp8"``: blocks of 32, power-of-two scale 2^ceil(log2(max(amax, 1e-4) / 448)), E4M3 values;
* ``"fp4_index"``: blocks of 32, power-of-two scale from max(amax, 6 * 2^-126) / 6, E2M1 values;
* ``"fp4_kv"``: blocks of 16, E4M3-rounded scale max(amax, 6 * 2^-9) / 6, E2M1 values.

E2M1 (magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6) rounds to nearest with ties to the even code. CUDA
tensors run ``csrc/fake_quant.cu``; the functions below are the CPU oracle.
"""

from __future__ import annotations

import torch

from ._ext import ext, on_gpu

KINDS = {"fp8": (0, 32), "fp4_index": (1, 32), "fp4_kv": (2, 16)}
_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _pow2_ceil(v: torch.Tensor) -> torch.Tensor:
    bits = v.contiguous().view(torch.int32)
    exponent = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    return torch.ldexp(torch.ones_like(v), exponent)


def _e2m1_round(v: torch.Tensor) -> torch.Tensor:
    a = v.abs()
    # the index of the grid value: thresholds at the midpoints, a tie goes to the even code
    index = ((a > 0.25).int() + (a >= 0.75).int() + (a > 1.25).int() + (a >= 1.75).int() + (a > 2.5).int()
             + (a >= 3.5).int() + (a > 5.0).int())
    magnitude = torch.tensor(_E2M1, dtype=torch.float32, device=v.device)[index.long()]
    return torch.where(torch.signbit(v), -magnitude, magnitude)


def fake_quant_reference(x: torch.Tensor, kind: str) -> torch.Tensor:
    code, block = KINDS[kind]
    if x.dim() == 0 or x.shape[-1] % block:
        return x
    blocks = x.float().reshape(*x.shape[:-1], x.shape[-1] // block, block)
    amax = blocks.abs().amax(-1, keepdim=True)
    if code == 0:
        scale = _pow2_ceil(amax.clamp_min(1e-4) / 448.0)
        q = (blocks / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float() * scale
    else:
        if code == 1:
            scale = _pow2_ceil(amax.clamp_min(6.0 * 2.0 ** -126) / 6.0)
        else:
            scale = (amax.clamp_min(6.0 * 2.0 ** -9) / 6.0).to(torch.float8_e4m3fn).float()
        q = _e2m1_round((blocks / scale).clamp(-6.0, 6.0)) * scale
    return q.reshape(x.shape).to(x.dtype)


def fake_quant(x: torch.Tensor, kind: str) -> torch.Tensor:
    if kind not in KINDS:
        raise ValueError(f"unknown quantization kind: {kind}")
    if on_gpu(x) and x.dtype in (torch.bfloat16, torch.float32):
        return ext().cache_fake_quant(x.contiguous(), KINDS[kind][0]).view_as(x)
    return fake_quant_reference(x, kind)


class _StraightThrough(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kind):
        return fake_quant(x.detach(), kind)

    @staticmethod
    def backward(ctx, grad):
        return grad, None


def quantize_activation(x: torch.Tensor, kind: str) -> torch.Tensor:
    return _StraightThrough.apply(x, kind)


__all__ = ["KINDS", "fake_quant", "fake_quant_reference", "quantize_activation"]
