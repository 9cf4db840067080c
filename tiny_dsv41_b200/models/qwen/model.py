"""Qwen3-MoE decoder for training on B200.

Parameter names and tensor layouts match ``dsv41_train/models/qwen/model.py`` (and therefore the
HF checkpoint after expert stacking): ``model.embed_tokens``, ``model.layers.N.self_attn.{q,k,v,o}_proj``,
``q_norm``/``k_norm``, ``mlp.gate``, ``mlp.experts.gate_up_proj [E_local, 2I, H]``,
``mlp.experts.down_proj [E_local, H, I]``, ``input_layernorm``, ``post_attention_layernorm``,
``model.norm``, ``lm_head``.

The hot path is built from the sm_100a ops: one fused QKV GEMM, fused per-head RMSNorm + RoPE,
tcgen05 grouped GEMMs over 128-row aligned expert segments (no per-expert Python loop, no host
synchronisation on one GPU), a fused router kernel that also carries the load-balancing
gradient, and a chunked LM-head cross entropy that never materialises full logits.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from ... import ops
from ...ops.router import AuxGradient
from ...parallel import replay
from ...parallel.cp import ContextParallel
from ...parallel.cp_attention import fused_supported
from ...parallel.dispatch import TokenDispatcher
from ...utils.trace import nvtx_range
from ..common import Linear, LMHead, fusable
from .config import Qwen3MoeConfig


class Qwen3MoeRMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(hidden, self.weight, self.variance_epsilon)


class Qwen3MoeAttention(nn.Module):
    def __init__(self, config: Qwen3MoeConfig, layer_id: int, context_parallel: ContextParallel) -> None:
        super().__init__()
        if config.head_dim != 128:
            raise ValueError("the fused QKV/RoPE kernel supports head_dim 128")
        self.layer_id = layer_id
        self.num_layers = config.num_hidden_layers
        self.context_parallel = context_parallel
        self.num_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        self.dropout = config.attention_dropout
        self.eps = config.rms_norm_eps
        self.rope_theta = config.rope_theta
        bias = config.attention_bias
        self.q_proj = Linear(config.hidden_size, self.num_heads * self.head_dim, bias=bias)
        self.k_proj = Linear(config.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = Linear(config.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.o_proj = Linear(self.num_heads * self.head_dim, config.hidden_size, bias=bias)
        self.q_norm = Qwen3MoeRMSNorm(self.head_dim, config.rms_norm_eps)
        self.k_norm = Qwen3MoeRMSNorm(self.head_dim, config.rms_norm_eps)

    def forward(self, hidden, position_ids, attention_mask=None, cache=None):
        batch, length, _ = hidden.shape
        freqs = ops.rope.cached_freqs(("rope", self.head_dim, self.rope_theta),
                                      ops.inv_freq(self.head_dim, self.rope_theta), hidden.device)
        if fusable(self.q_proj, self.k_proj, self.v_proj):
            weight = torch.cat((self.q_proj.weight, self.k_proj.weight, self.v_proj.weight), dim=0)
            qkv = ops.linear(hidden, weight, replayable=True)  # the recompute reuses this product
        else:
            qkv = torch.cat((self.q_proj(hidden), self.k_proj(hidden), self.v_proj(hidden)), dim=-1)
        q, k, v = ops.qk_norm_rope(qkv, self.q_norm.weight, self.k_norm.weight, position_ids, freqs,
                                   self.num_heads, self.num_key_value_heads, self.eps)
        q = q.view(batch, length, self.num_heads, self.head_dim)
        k = k.view(batch, length, self.num_key_value_heads, self.head_dim)
        v = v.reshape(batch, length, self.num_key_value_heads, self.head_dim)
        cp = self.context_parallel
        mask = None
        if cache is not None:  # incremental decoding: attend over cached keys/values of earlier positions
            if cp.enabled:
                raise ValueError("the KV cache does not support context parallelism")
            k, v, key_positions = cache.append(self.layer_id, k, v, position_ids)
            mask = key_positions[:, None, None, :] <= position_ids[:, None, :, None]
            out = ops.causal_attention(q, k, v, mask=mask)
            return self.o_proj(out.reshape(batch, length, -1))
        if cp.enabled and cp.fused_attention and cp.plain_causal and attention_mask is None and \
                fused_supported(q, k, cp.size):
            # K/V chunks of the other CP ranks stream over NVLink into the attention kernels
            out = cp.fused(self.num_layers)(q, k, v, self.layer_id)
            return self.o_proj(out.reshape(batch, length, -1))
        if cp.enabled:
            k = cp.gather(k, dim=1)
            v = cp.gather(v, dim=1)
            key_positions = cp.gather(position_ids, dim=1)
            mask = key_positions[:, None, None, :] <= position_ids[:, None, :, None]
            if attention_mask is not None:
                valid = cp.gather(attention_mask, dim=1).bool()
                mask = mask & valid[:, None, None, :]
        elif attention_mask is not None:
            causal = torch.ones(length, length, dtype=torch.bool, device=hidden.device).tril()
            mask = causal.view(1, 1, length, length) & attention_mask.bool()[:, None, None, :]
        out = ops.causal_attention(q, k, v, mask=mask, dropout=self.dropout if self.training else 0.0)
        if fusable(self.o_proj):
            return ops.linear(out.reshape(batch, length, -1), self.o_proj.weight, replayable=True)
        return self.o_proj(out.reshape(batch, length, -1))


class Qwen3MoeMLP(nn.Module):
    def __init__(self, config: Qwen3MoeConfig, intermediate_size: int | None = None) -> None:
        super().__init__()
        size = config.intermediate_size if intermediate_size is None else intermediate_size
        self.gate_proj = Linear(config.hidden_size, size, bias=False)
        self.up_proj = Linear(config.hidden_size, size, bias=False)
        self.down_proj = Linear(size, config.hidden_size, bias=False)

    def forward(self, hidden):
        if fusable(self.gate_proj, self.up_proj):
            gu = ops.linear(hidden, torch.cat((self.gate_proj.weight, self.up_proj.weight), dim=0))
        else:
            gu = torch.cat((self.gate_proj(hidden), self.up_proj(hidden)), dim=-1)
        return self.down_proj(ops.swiglu(gu.reshape(-1, gu.shape[-1])).view(*hidden.shape[:-1], -1))


class Qwen3MoeExperts(nn.Module):
    """This EP rank's experts, stacked; routed through the dispatcher's expert-major layout."""

    def __init__(self, config: Qwen3MoeConfig, dispatcher: TokenDispatcher) -> None:
        super().__init__()
        self.dispatcher = dispatcher
        self.global_num_experts = config.num_experts
        self.expert_start, stop = dispatcher.expert_range(config.num_experts)
        self.num_experts = stop - self.expert_start
        self.intermediate_size = config.moe_intermediate_size
        self.gate_up_proj = nn.Parameter(torch.empty(self.num_experts, 2 * config.moe_intermediate_size,
                                                     config.hidden_size))
        self.down_proj = nn.Parameter(torch.empty(self.num_experts, config.hidden_size,
                                                  config.moe_intermediate_size))

    def forward(self, hidden, selected_experts, weights):
        batch = self.dispatcher.dispatch(hidden, selected_experts, weights)
        gate_up = ops.grouped_linear(batch.rows, self.gate_up_proj, batch.offsets, batch.sizes)
        act = ops.swiglu(gate_up, total=batch.total)
        out = ops.grouped_linear(act, self.down_proj, batch.offsets, batch.sizes)
        return self.dispatcher.combine(out, batch, weighted=True)


class Qwen3MoeSparseMoeBlock(nn.Module):
    def __init__(self, config: Qwen3MoeConfig, dispatcher: TokenDispatcher) -> None:
        super().__init__()
        self.num_experts = config.num_experts
        self.top_k = config.num_experts_per_tok
        self.norm_topk_prob = config.norm_topk_prob
        self.gate = Linear(config.hidden_size, config.num_experts, bias=False)
        self.experts = Qwen3MoeExperts(config, dispatcher)
        self.aux: AuxGradient | None = None
        self.stats: list | None = None

    def forward(self, hidden):
        batch, length, size = hidden.shape
        flat = hidden.reshape(-1, size)
        router_logits = self.gate(flat)
        selected, weights = ops.route(router_logits, self.top_k, func="softmax", normalize=self.norm_topk_prob,
                                      aux=self.aux)
        if self.stats is not None:
            with torch.no_grad():
                probs = torch.softmax(router_logits.float(), dim=-1)
                # scatter-add instead of bincount, which reads the maximum back to the host
                ids = selected.reshape(-1).long()
                counts = torch.zeros(self.num_experts, dtype=torch.long, device=ids.device).scatter_add_(
                    0, ids, torch.ones_like(ids))
                self.stats.append((counts.float(), probs.sum(0), probs.shape[0]))
        out = self.experts(flat, selected, weights)
        return out.reshape(batch, length, size), router_logits


class Qwen3MoeDecoderLayer(nn.Module):
    def __init__(self, config, layer_id, context_parallel, dispatcher) -> None:
        super().__init__()
        self.self_attn = Qwen3MoeAttention(config, layer_id, context_parallel)
        self.mlp = (Qwen3MoeSparseMoeBlock(config, dispatcher) if config.is_sparse_layer(layer_id)
                    else Qwen3MoeMLP(config, config.intermediate_size))
        self.input_layernorm = Qwen3MoeRMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = Qwen3MoeRMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, hidden, position_ids, attention_mask=None, cache=None):
        with nvtx_range("attention"):
            hidden = hidden + self.self_attn(self.input_layernorm(hidden), position_ids, attention_mask, cache)
        with nvtx_range("moe"):
            out = self.mlp(self.post_attention_layernorm(hidden))
        logits = None
        if isinstance(out, tuple):
            out, logits = out
        return hidden + out, logits


@dataclass
class Qwen3MoeModelOutput:
    last_hidden_state: torch.Tensor
    router_logits: tuple[torch.Tensor, ...] | None


class Qwen3MoeModel(nn.Module):
    def __init__(self, config, context_parallel=None, token_dispatcher=None) -> None:
        super().__init__()
        self.config = config
        self.context_parallel = context_parallel or ContextParallel()
        token_dispatcher = token_dispatcher or TokenDispatcher()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(Qwen3MoeDecoderLayer(config, i, self.context_parallel, token_dispatcher)
                                    for i in range(config.num_hidden_layers))
        self.norm = Qwen3MoeRMSNorm(config.hidden_size, config.rms_norm_eps)
        self.gradient_checkpointing = False

    def forward(self, input_ids, attention_mask=None, position_ids=None, *, output_router_logits=False, cache=None):
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [batch, sequence]")
        if input_ids.shape[1] > self.config.max_position_embeddings:
            raise ValueError("sequence is longer than max_position_embeddings")
        if attention_mask is not None and attention_mask.shape != input_ids.shape:
            raise ValueError("attention_mask must have the same shape as input_ids")
        cp = self.context_parallel
        cp.plain_causal = position_ids is None and attention_mask is None and cache is None
        if position_ids is None:
            position_ids = torch.arange(input_ids.shape[1], device=input_ids.device).unsqueeze(0).expand_as(input_ids)
        input_ids, position_ids = cp.shard(input_ids), cp.shard(position_ids.contiguous())
        if attention_mask is not None:
            attention_mask = cp.shard(attention_mask)
        hidden = self.embed_tokens(input_ids)
        collected = []
        for layer in self.layers:
            if cache is not None:
                hidden, logits = layer(hidden, position_ids, attention_mask, cache)
            elif self.gradient_checkpointing and self.training and torch.is_grad_enabled():
                # the RNG state matters only with dropout (and reading it is not allowed in a CUDA-graph capture)
                hidden, logits = checkpoint(layer, hidden, position_ids, attention_mask, use_reentrant=False,
                                            context_fn=replay.checkpoint_contexts,
                                            preserve_rng_state=self.config.attention_dropout > 0)
            else:
                hidden, logits = layer(hidden, position_ids, attention_mask)
            if output_router_logits and logits is not None:
                collected.append(logits)
        return Qwen3MoeModelOutput(self.norm(hidden), tuple(collected) if output_router_logits else None)


@dataclass
class Qwen3MoeCausalLMOutput:
    loss: torch.Tensor | None
    logits: torch.Tensor | None
    aux_loss: torch.Tensor | None
    router_logits: tuple[torch.Tensor, ...] | None


class Qwen3MoeForCausalLM(nn.Module):
    def __init__(self, config: Qwen3MoeConfig, context_parallel=None, token_dispatcher=None) -> None:
        super().__init__()
        self.config = config
        self.context_parallel = context_parallel or ContextParallel()
        self.model = Qwen3MoeModel(config, self.context_parallel, token_dispatcher)
        self.lm_head = LMHead(config.hidden_size, config.vocab_size)
        self.aux_gradient = AuxGradient()
        for module in self.modules():
            if isinstance(module, Qwen3MoeSparseMoeBlock):
                module.aux = self.aux_gradient
        self.apply(self._initialize)

    def _initialize(self, module: nn.Module) -> None:
        std = self.config.initializer_range
        if any(p.is_meta for p in module.parameters(recurse=False)):
            return
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=std)
            if getattr(module, "bias", None) is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, Qwen3MoeExperts):
            nn.init.normal_(module.gate_up_proj, mean=0.0, std=std)
            nn.init.normal_(module.down_proj, mean=0.0, std=std)
        elif isinstance(module, Qwen3MoeRMSNorm):
            nn.init.ones_(module.weight)

    def gradient_checkpointing_enable(self) -> None:
        self.model.gradient_checkpointing = True

    def _moe_blocks(self):
        return [m for m in self.modules() if isinstance(m, Qwen3MoeSparseMoeBlock)]

    def forward(self, input_ids, attention_mask=None, labels=None, *, position_ids=None, output_router_logits=None):
        output_router_logits = self.config.output_router_logits if output_router_logits is None else output_router_logits
        blocks = self._moe_blocks()
        stats: list = []
        for block in blocks:
            block.stats = stats if output_router_logits else None
        self.aux_gradient.set(None)
        try:
            output = self.model(input_ids, attention_mask, position_ids, output_router_logits=output_router_logits)
        finally:
            for block in blocks:
                block.stats = None
        hidden = output.last_hidden_state
        cp = self.context_parallel
        loss = logits = None
        aux_loss = None
        if output_router_logits and stats:
            aux_loss = self._aux_loss(stats, attention_mask)
        if labels is not None:
            targets = torch.full_like(labels, -100)
            targets[:, :-1] = labels[:, 1:]
            if attention_mask is not None:
                targets[:, :-1].masked_fill_(~attention_mask[:, 1:].bool(), -100)
            targets = cp.shard(targets)
            loss_sum = self.lm_head(hidden, targets, mode="ce_sum")
            loss = cp.mean_loss(loss_sum, (targets != -100).sum())
            if aux_loss is not None:
                loss = loss + self.config.router_aux_loss_coef * aux_loss.detach()
        else:
            logits = self.lm_head(hidden)
        return Qwen3MoeCausalLMOutput(loss, logits, aux_loss, output.router_logits)

    def _aux_loss(self, stats, attention_mask):
        """E * sum_e f_e * P_e over all layers' tokens; its gradient is injected in the router backward."""
        experts = self.config.num_experts
        counts = torch.stack([c for c, _, _ in stats]).sum(0)
        psum = torch.stack([p for _, p, _ in stats]).sum(0)
        total = counts.new_full((), float(sum(n for _, _, n in stats)), dtype=torch.float32)  # no host copy
        cp = self.context_parallel
        counts, psum, total = cp.sum(counts), cp.sum(psum), cp.sum(total)
        aux = experts * ((counts / total) * (psum / total)).sum()
        coef = self.config.router_aux_loss_coef
        if torch.is_grad_enabled() and coef:
            # d(coef * aux) / d softmax_{t,e} for one token of one layer (times CP scale so that
            # FSDP's average over ranks yields the global gradient).
            self.aux_gradient.set(coef * experts * counts / (total * total) * cp.size)
        return aux


__all__ = [
    "Qwen3MoeAttention", "Qwen3MoeCausalLMOutput", "Qwen3MoeDecoderLayer", "Qwen3MoeExperts",
    "Qwen3MoeForCausalLM", "Qwen3MoeMLP", "Qwen3MoeModel", "Qwen3MoeModelOutput", "Qwen3MoeRMSNorm",
    "Qwen3MoeSparseMoeBlock",
]
