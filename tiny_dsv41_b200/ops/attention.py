"""Causal GQA attention for Qwen3 (``dsv41_train/models/qwen/model.py:84-171``).

Layout: q [B, L, Hq, D], k/v [B, L, Hkv, D] (the token-major layout the QKV kernel writes).
This entry point runs PyTorch's scaled-dot-product attention (a library kernel: cuDNN's fused
attention on B200). No attention kernel of this library exists yet; every model calls attention
through this function so one can replace it in a single place.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, mask: torch.Tensor | None = None,
                     dropout: float = 0.0) -> torch.Tensor:
    """Returns [B, L, Hq, D]. ``mask`` (optional) is a boolean [B, 1, Lq, Lk] keep-mask."""
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
