"""Causal GQA attention for Qwen3 (``dsv41_train/models/qwen/model.py:84-171``; the reference calls
``F.scaled_dot_product_attention`` at line 162).

Layout: q [B, L, Hq, D], k/v [B, L, Hkv, D] (the token-major layout the QKV kernel writes).
On CUDA, the plain causal case (no extra mask, no dropout, bf16, head dim 128, L a multiple of
128) runs this library's tcgen05 flash-attention kernels (``csrc/attention.cu``): forward
saves (out, lse), backward recomputes P per tile; under activation checkpointing the recompute
reuses the first pass's (out, lse) (``parallel/replay.py``) instead of running the forward again. Anything else (an explicit mask for padding,
context parallelism or a KV cache; dropout; other shapes) runs PyTorch's scaled-dot-product
attention, as do CPU tensors (the numerical oracle).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v):
        from ..parallel import replay

        handle, mode = replay.current()
        if mode == "replay":  # checkpoint recompute: the first pass's result (same inputs, same kernel)
            out, lse = handle.next_attention()
            out = out.clone()  # a fresh output: the record must not become this node's output
        else:
            out, lse = ext().attn_fwd(q, k, v)
            if mode == "record":
                handle.record_attention((out.detach(), lse))
        ctx.save_for_backward(q, k, v, out, lse)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = ext().attn_bwd(dout.contiguous(), q, k, v, out, lse)
        return dq, dk, dv


def flash_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    return (q.dtype == torch.bfloat16 and k.dtype == q.dtype and v.dtype == q.dtype and q.shape[-1] == 128
            and q.shape[1] % 128 == 0 and q.shape[1] > 0 and k.shape[1] == q.shape[1]
            and q.shape[2] % k.shape[2] == 0)


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal attention through the tcgen05 kernels (CUDA, bf16, head dim 128, L % 128 == 0)."""
    return _FlashAttention.apply(q.contiguous(), k.contiguous(), v.contiguous())


def sdpa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, mask: torch.Tensor | None = None,
                   dropout: float = 0.0) -> torch.Tensor:
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    groups = qh.shape[1] // kh.shape[1]
    if mask is None:
        out = F.scaled_dot_product_attention(qh, kh, vh, dropout_p=dropout, is_causal=True,
                                             enable_gqa=groups > 1)
    else:
        if groups > 1:
            kh = kh.repeat_interleave(groups, dim=1)
            vh = vh.repeat_interleave(groups, dim=1)
        out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, dropout_p=dropout)
    return out.transpose(1, 2)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, mask: torch.Tensor | None = None,
                     dropout: float = 0.0) -> torch.Tensor:
    """Returns [B, L, Hq, D]. ``mask`` (optional) is a boolean [B, 1, Lq, Lk] keep-mask."""
    if mask is None and dropout == 0.0 and on_gpu(q) and flash_supported(q, k, v):
        return flash_attention(q, k, v)
    return sdpa_attention(q, k, v, mask=mask, dropout=dropout)
