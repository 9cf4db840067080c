"""Rotary embeddings.

* ``qk_norm_rope``: Qwen3 per-head q/k RMSNorm + rotate-half RoPE fused over the packed QKV
  projection output (``dsv41_train/models/qwen/model.py:19-35, 114-123``).
* ``rope_interleaved``: DSV4 even/odd rotation of the last ``rope_dim`` channels, forward or
  inverse (``dsv41_train/models/dsv4/attention/module.py:72-85``).
"""

from __future__ import annotations

import torch

from ._ext import ext, on_gpu
from .norm import rms_norm_reference


def inv_freq(dim: int, theta: float, device=None) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim))


_FREQ_CACHE: dict = {}


def cached_freqs(key, values: torch.Tensor, device) -> torch.Tensor:
    """fp32 frequency table on `device`, kept outside module buffers so that dtype casts of the
    model (``.to(bfloat16)``, FSDP mixed-precision input casts) never touch it."""
    device = torch.device(device)
    full = (key, str(device))
    table = _FREQ_CACHE.get(full)
    if table is None:
        table = values.detach().to(device=device, dtype=torch.float32).contiguous()
        _FREQ_CACHE[full] = table
    return table


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def qk_norm_rope_reference(qkv, wq, wk, positions, freqs, hq, hkv, eps):
    d = 128
    tokens = qkv.reshape(-1, qkv.shape[-1])
    q, k, v = tokens.split([hq * d, hkv * d, hkv * d], dim=-1)
    q = rms_norm_reference(q.reshape(-1, hq, d), wq, eps)
    k = rms_norm_reference(k.reshape(-1, hkv, d), wk, eps)
    angles = positions.reshape(-1).float().unsqueeze(-1) * freqs.float()
    emb = torch.cat((angles, angles), dim=-1)
    cos, sin = emb.cos().unsqueeze(1), emb.sin().unsqueeze(1)
    qo = (q.float() * cos + _rotate_half(q.float()) * sin).to(qkv.dtype)
    ko = (k.float() * cos + _rotate_half(k.float()) * sin).to(qkv.dtype)
    return qo, ko, v.reshape(-1, hkv, d)


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, wq, wk, positions, freqs, hq, hkv, eps):
        from ..parallel import replay

        qkv2 = qkv.reshape(-1, qkv.shape[-1]).contiguous()
        pos = positions.reshape(-1).contiguous()
        handle, mode = replay.current()
        if mode == "replay":  # checkpoint recompute: the first pass's q / k (same inputs)
            q, k = (t.clone() for t in handle.next_attention())
        else:
            q, k = ext().qk_norm_rope_fwd(qkv2, wq.contiguous(), wk.contiguous(), pos, freqs, hq, hkv, float(eps))
            if mode == "record":
                handle.record_attention((q.detach(), k.detach()))
        ctx.save_for_backward(qkv2, wq, wk, pos, freqs)
        ctx.meta = (hq, hkv, eps, qkv.shape)
        v = qkv2[:, (hq + hkv) * 128:].view(-1, hkv, 128)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv2, wq, wk, pos, freqs = ctx.saved_tensors
        hq, hkv, eps, shape = ctx.meta
        dq = torch.zeros_like(qkv2[:, : hq * 128]).view(-1, hq, 128) if dq is None else dq.contiguous()
        dk = torch.zeros(qkv2.shape[0], hkv, 128, dtype=qkv2.dtype, device=qkv2.device) if dk is None else dk.contiguous()
        dv = torch.zeros(qkv2.shape[0], hkv, 128, dtype=qkv2.dtype, device=qkv2.device) if dv is None else dv.contiguous()
        dqkv, dwq, dwk = ext().qk_norm_rope_bwd(dq, dk, dv, qkv2, wq.contiguous(), wk.contiguous(), pos, freqs,
                                                hq, hkv, float(eps))
        return dqkv.view(shape), dwq.to(wq.dtype), dwk.to(wk.dtype), None, None, None, None, None


def qk_norm_rope(qkv, wq, wk, positions, freqs, hq: int, hkv: int, eps: float):
    """Returns q [T, hq, 128], k [T, hkv, 128], v [T, hkv, 128] from qkv [..., (hq+2hkv)*128]."""
    if on_gpu(qkv) and qkv.dtype == torch.bfloat16:
        return _QKNormRope.apply(qkv, wq, wk, positions, freqs, hq, hkv, eps)
    return qk_norm_rope_reference(qkv, wq, wk, positions, freqs, hq, hkv, eps)


def rope_interleaved_reference(x, positions, freqs, rope_dim, inverse=False):
    angles = positions.reshape(-1).float().unsqueeze(-1) * freqs.float()
    cos, sin = angles.cos(), angles.sin()
    if inverse:
        sin = -sin
    plain, rotary = x[..., :-rope_dim], x[..., -rope_dim:]
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    even, odd = rotary[..., 0::2].float(), rotary[..., 1::2].float()
    rotary = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(-2)
    return torch.cat((plain, rotary.to(x.dtype)), dim=-1)


class _RopeInterleaved(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, positions, freqs, rope_dim, inverse):
        pos = positions.reshape(-1).contiguous()
        ctx.save_for_backward(pos, freqs)
        ctx.meta = (rope_dim, inverse)
        return ext().rope_interleaved(x.contiguous(), pos, freqs, rope_dim, inverse)

    @staticmethod
    def backward(ctx, dy):
        pos, freqs = ctx.saved_tensors
        rope_dim, inverse = ctx.meta
        return ext().rope_interleaved(dy.contiguous(), pos, freqs, rope_dim, not inverse), None, None, None, None


def rope_interleaved(x, positions, freqs, rope_dim: int, inverse: bool = False):
    """x: [rows, heads, D]; positions: [rows]."""
    if on_gpu(x) and x.dtype == torch.bfloat16:
        return _RopeInterleaved.apply(x, positions, freqs, rope_dim, inverse)
    return rope_interleaved_reference(x, positions, freqs, rope_dim, inverse)
