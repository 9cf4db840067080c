"""DeepSeek-V4.1 sparse MoE: biased top-k router, routed experts with clamped SwiGLU, shared expert.

Parameter names/layouts follow ``dsv41_train/models/dsv4/moe/module.py``: ``router.weight [E, H]``,
``router.selection_bias`` (buffer), ``routed.gate_up [E_local, I, 2, H]`` (gate/up interleaved per
intermediate column), ``routed.down [E_local, H, I]``, ``shared.{gate,up,down}``.
The routed path runs on the tcgen05 grouped GEMMs over the dispatcher's expert-major segments; the
route weight multiplies inside the clamped SwiGLU, as in the reference.
"""

from __future__ import annotations

import torch
from torch import nn

from ... import ops
from ...ops.router import AuxGradient
from ...parallel.dispatch import TokenDispatcher
from ..common import Linear, fusable
from .config import DeepSeekV41Config


class TopKRouter(nn.Module):
    def __init__(self, config: DeepSeekV41Config) -> None:
        super().__init__()
        self.topk = config.num_experts_per_tok
        self.num_experts = config.n_routed_experts
        self.score_name = config.scoring_func
        self.temperature = config.gate_temp
        self.normalize = config.norm_topk_prob
        self.scale = config.routed_scaling_factor
        self.weight = nn.Parameter(torch.empty(self.num_experts, config.hidden_size))
        self.register_buffer("selection_bias", torch.zeros(self.num_experts))
        self.aux: AuxGradient | None = None

    def forward(self, x: torch.Tensor):
        logits = torch.nn.functional.linear(x.flatten(0, 1).float(), self.weight.float()) / self.temperature
        indices, weights = ops.route(logits, self.topk, func=self.score_name, bias=self.selection_bias.float(),
                                     normalize=self.normalize, norm_eps=1e-20, scale=self.scale, aux=self.aux)
        return logits, weights, indices


class RoutedExperts(nn.Module):
    def __init__(self, config: DeepSeekV41Config, dispatcher: TokenDispatcher) -> None:
        super().__init__()
        self.dispatcher = dispatcher
        self.global_num_experts = config.n_routed_experts
        self.expert_start, stop = dispatcher.expert_range(config.n_routed_experts)
        self.num_experts = stop - self.expert_start
        self.hidden_size = config.hidden_size
        self.intermediate = config.moe_intermediate_size
        self.limit = config.swiglu_limit
        self.gate_up = nn.Parameter(torch.empty(self.num_experts, self.intermediate, 2, self.hidden_size))
        self.down = nn.Parameter(torch.empty(self.num_experts, self.hidden_size, self.intermediate))

    @property
    def local_parameter_count(self) -> int:
        if self.frozen_fp4:
            return 2 * (self.gate_up_fp4.numel() + self.down_fp4.numel())
        return self.gate_up.numel() + self.down.numel()

    @property
    def frozen_fp4(self) -> bool:
        return "gate_up_fp4" in self._buffers

    def freeze_fp4(self, gate_up_fp4, gate_up_scale, down_fp4, down_scale) -> None:
        """Replace the bf16 expert weights by frozen MXFP4 codes and E8M0 scales (uint8):
        gate_up [E, I, 2, H/2] / [E, I, 2, H/32], down [E, H, I/2] / [E, H, I/32]. The grouped
        GEMMs read them packed and they are never trained (LoRA SFT over a released FP4
        checkpoint)."""
        e, i, h = self.num_experts, self.intermediate, self.hidden_size
        shapes = ((gate_up_fp4, (e, i, 2, h // 2)), (gate_up_scale, (e, i, 2, h // 32)),
                  (down_fp4, (e, h, i // 2)), (down_scale, (e, h, i // 32)))
        if any(t.dtype != torch.uint8 or tuple(t.shape) != s for t, s in shapes):
            raise ValueError("frozen FP4 experts need uint8 codes and scales of the expert shapes")
        del self.gate_up, self.down
        for name, (t, _) in zip(("gate_up_fp4", "gate_up_scale", "down_fp4", "down_scale"), shapes):
            self.register_buffer(name, t)

    def forward(self, x, indices, weights):
        batch = self.dispatcher.dispatch(x, indices, weights)
        row_weights = self.dispatcher.row_weights(batch)
        if self.frozen_fp4:
            e, i, h = self.num_experts, self.intermediate, self.hidden_size
            gate_up = ops.fp4_grouped_linear(batch.rows, self.gate_up_fp4.view(e, 2 * i, h // 2),
                                             self.gate_up_scale.view(e, 2 * i, h // 32), batch.offsets, batch.sizes,
                                             2 * i)
        else:
            w1 = self.gate_up.reshape(self.num_experts, 2 * self.intermediate, self.hidden_size)
            gate_up = ops.grouped_linear(batch.rows, w1, batch.offsets, batch.sizes)
        hidden = ops.swiglu(gate_up, row_weights, interleaved=True, limit=self.limit, total=batch.total)
        if self.frozen_fp4:
            out = ops.fp4_grouped_linear(hidden, self.down_fp4, self.down_scale, batch.offsets, batch.sizes,
                                         self.hidden_size)
        else:
            out = ops.grouped_linear(hidden, self.down, batch.offsets, batch.sizes)
        return self.dispatcher.combine(out, batch, weighted=False)


class SharedExpert(nn.Module):
    def __init__(self, config: DeepSeekV41Config) -> None:
        super().__init__()
        inter = config.moe_intermediate_size * config.n_shared_experts
        self.gate = Linear(config.hidden_size, inter, bias=False)
        self.up = Linear(config.hidden_size, inter, bias=False)
        self.down = Linear(inter, config.hidden_size, bias=False)
        self.limit = config.swiglu_limit

    def forward(self, x):
        if fusable(self.gate, self.up):
            gu = ops.linear(x, torch.cat((self.gate.weight, self.up.weight), dim=0))
        else:
            gu = torch.cat((self.gate(x), self.up(x)), dim=-1)
        hidden = ops.swiglu(gu.reshape(-1, gu.shape[-1]), limit=self.limit).view(*x.shape[:-1], -1)
        return self.down(hidden.to(x.dtype))


class SparseMoE(nn.Module):
    def __init__(self, config: DeepSeekV41Config, dispatcher: TokenDispatcher) -> None:
        super().__init__()
        self.router = TopKRouter(config)
        self.routed = RoutedExperts(config, dispatcher)
        self.shared = SharedExpert(config)

    def forward(self, x: torch.Tensor):
        shape = x.shape
        flat = x.flatten(0, 1)
        logits, weights, indices = self.router(x)
        out = self.routed(flat, indices, weights).float() + self.shared(flat).float()
        return out.to(x.dtype).view(shape), logits


__all__ = ["RoutedExperts", "SharedExpert", "SparseMoE", "TopKRouter"]
