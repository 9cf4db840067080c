"""mHC hyper-connection for DeepSeek-V4.1 (4 residual streams).

Parameters ``fn [(2+hc)*hc, hc*H]``, ``base [(2+hc)*hc]``, ``scale [3]`` (fp32 islands), as in
``dsv41_train/models/dsv4/mhc.py:524-565``. ``forward(streams, input_weights)`` RMS-normalises
the concatenated streams, projects to (pre, post, comb) mixing logits, and returns the branch
input collapsed with the *incoming* weights plus the new (pre, post, comb); ``finish`` expands
the branch output back into the streams.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ...ops import mhc as mhc_ops
from .config import DeepSeekV41Config


def mixing_weights(projected, base, scale, hc: int, iterations: int, eps: float):
    pre, post, comb = projected.float().split([hc, hc, hc * hc], dim=-1)
    pre_bias, post_bias, comb_bias = base.float().split([hc, hc, hc * hc])
    pre_scale, post_scale, comb_scale = scale.float()
    pre = torch.sigmoid(pre * pre_scale + pre_bias) + eps
    post = 2 * torch.sigmoid(post * post_scale + post_bias)
    comb = comb.view(*comb.shape[:-1], hc, hc) * comb_scale + comb_bias.view(hc, hc)
    comb = mhc_ops.sinkhorn(comb, iterations, eps)
    return pre, post, comb


class HyperConnection(nn.Module):
    def __init__(self, config: DeepSeekV41Config) -> None:
        super().__init__()
        self.hc_mult = config.hc_mult
        self.sinkhorn_iters = config.hc_sinkhorn_iters
        self.eps = config.hc_eps
        mix = (2 + config.hc_mult) * config.hc_mult
        self.fn = nn.Parameter(torch.empty(mix, config.hc_mult * config.hidden_size))
        self.base = nn.Parameter(torch.zeros(mix))
        self.scale = nn.Parameter(torch.ones(3))
        self.norm_eps = config.rms_norm_eps

    def forward(self, streams: torch.Tensor, input_weights: torch.Tensor):
        flat = streams.flatten(2).float()
        flat = flat * torch.rsqrt(flat.square().mean(-1, keepdim=True) + self.norm_eps)
        projected = F.linear(flat, self.fn.float())
        pre, post, comb = mixing_weights(projected, self.base, self.scale, self.hc_mult, self.sinkhorn_iters, self.eps)
        return mhc_ops.collapse(streams, input_weights), pre, post, comb

    @staticmethod
    def finish(value, residual, output_weights, residual_weights):
        return mhc_ops.expand(value, residual, output_weights, residual_weights)

    @staticmethod
    def collapse(streams, weights):
        return mhc_ops.collapse(streams, weights)


__all__ = ["HyperConnection", "mixing_weights"]
