"""DeepSeek-V4.1 CSA2 attention: low-rank query, one shared 512-wide KV head with sliding-window
keys, compressed global KV latents chosen by a sparse indexer, learned per-head sink logits and a
grouped low-rank output projection.

Module structure and parameter names follow ``dsv41_train/models/dsv4/attention/module.py``
(``CSA2Attention`` 350-471, ``Compressor`` 125-197, ``SparseIndexer`` 227-347); the attention
itself is :func:`tiny_dsv41_b200.ops.sparse_attention.sparse_attention`.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...ops.quant import quantize_activation
from ...ops.sparse_attention import index_scores, sparse_attention
from ...parallel.cp import ModelContext
from ..common import Linear
from .config import DeepSeekV41Config


class RMSNorm(nn.Module):
    def __init__(self, size: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)


class RotaryEmbedding(nn.Module):
    """Two inverse-frequency sets: main (rope_theta) and compressed (compress_rope_theta, YaRN)."""

    def __init__(self, config: DeepSeekV41Config) -> None:
        super().__init__()
        dim = config.qk_rope_head_dim
        self.dim = dim
        # computed on the host even under a meta-device context: these are constants, not weights
        main = 1.0 / (config.rope_theta ** (torch.arange(0, dim, 2, device="cpu").float() / dim))
        compressed = 1.0 / (config.compress_rope_theta ** (torch.arange(0, dim, 2, device="cpu").float() / dim))
        scaling = config.rope_scaling or {}
        if scaling.get("rope_type", scaling.get("type")) == "yarn":
            factor = scaling["factor"]
            original = scaling["original_max_position_embeddings"]
            beta_fast = scaling.get("beta_fast", 32)
            beta_slow = scaling.get("beta_slow", 1)

            def corrected(rotations: float) -> float:
                return dim * math.log(original / (rotations * 2 * math.pi)) / (2 * math.log(config.compress_rope_theta))

            low = max(math.floor(corrected(beta_fast)), 0)
            high = min(math.ceil(corrected(beta_slow)), dim - 1)
            ramp = ((torch.arange(dim // 2, dtype=torch.float32, device="cpu") - low) / max(high - low, 1e-3)).clamp(0, 1)
            keep = 1 - ramp
            compressed = compressed / factor * (1 - keep) + compressed * keep
        self.register_buffer("main", main.to(torch.empty(0).device), persistent=False)
        self.register_buffer("compressed", compressed.to(torch.empty(0).device), persistent=False)
        # fp32 copies outside the buffers: model dtype casts must not round the frequencies
        self._main_fp32, self._compressed_fp32 = main.clone(), compressed.clone()
        self._key = (dim, config.rope_theta, config.compress_rope_theta, repr(sorted(scaling.items())))

    def freqs(self, compressed: bool, device=None) -> torch.Tensor:
        device = self.main.device if device is None else device
        values = self._compressed_fp32 if compressed else self._main_fp32
        return ops.rope.cached_freqs(("dsv4", compressed, self._key), values, device)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, *, inverse: bool = False) -> torch.Tensor:
    """Interleaved rotation of the last ``2*len(freqs)`` channels. x: [B, L, (H,) D]; positions [B, L]."""
    shape = x.shape
    heads = shape[2] if x.ndim == 4 else 1
    rows = x.reshape(shape[0] * shape[1], heads, shape[-1])
    out = ops.rope_interleaved(rows, positions.reshape(-1), freqs, 2 * freqs.shape[0], inverse)
    return out.view(shape)


class GroupedLinear(nn.Module):
    def __init__(self, input_per_group: int, output_per_group: int, groups: int) -> None:
        super().__init__()
        self.groups = groups
        self.weight = nn.Parameter(torch.empty(groups, output_per_group, input_per_group))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-2]
        grouped = x.reshape(-1, self.groups, x.shape[-1]).transpose(0, 1)
        out = torch.bmm(grouped, self.weight.transpose(1, 2).to(x.dtype)).transpose(0, 1)
        return out.reshape(*lead, self.groups, -1)


class AttentionSinks(nn.Module):
    """fp32 per-head sink logits."""

    def __init__(self, num_heads: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(num_heads))

    def forward(self, reference: torch.Tensor | None = None) -> torch.Tensor:
        return self.weight.clone()


class CSA2Mode(str, Enum):
    FULL = "full"
    REINDEX = "reindex"
    REUSE = "reuse"


def complete_group_starts(positions: torch.Tensor, live: torch.Tensor, sequence_ids: torch.Tensor, ratio: int):
    """Token index of the first member of every complete compression group, packed to the left of
    each row ([B, L // ratio], unused slots 0), and the number of groups per row.

    A group opens at a live token whose position is a multiple of ``ratio`` and is complete when
    its last member (``ratio - 1`` tokens later) exists, is live and belongs to the same sequence
    (packed rows hold several sequences)."""
    batch, length = positions.shape
    token = torch.arange(length, device=positions.device)
    last = token + ratio - 1
    last_row = last.clamp_max(length - 1).expand(batch, -1)
    opens = live & (positions % ratio == 0) & (last < length)
    opens = opens & live.gather(1, last_row) & (sequence_ids == sequence_ids.gather(1, last_row))
    slot = torch.where(opens, opens.long().cumsum(-1) - 1, length)  # closed groups go to a spare column
    packed = positions.new_zeros(batch, length + 1).scatter_(1, slot, token.expand(batch, -1))
    return packed[:, :length // ratio], opens.sum(-1)


class Compressor(nn.Module):
    """Pools complete groups of `ratio` live tokens into global KV latents (a softmax-gated
    weighted sum of the group's projections when ratio > 1, the projection itself otherwise)."""

    def __init__(self, config: DeepSeekV41Config, layer_id: int) -> None:
        super().__init__()
        self.ratio = config.compress_ratios[layer_id]
        self.kv_proj = Linear(config.hidden_size, config.head_dim, bias=False)
        self.gate_proj = Linear(config.hidden_size, config.head_dim, bias=False) if self.ratio > 1 else None
        self.norm = RMSNorm(config.head_dim, config.rms_norm_eps)

    def forward(self, x, positions, token_mask, sequence_ids):
        starts, count = complete_group_starts(positions, token_mask.bool(), sequence_ids, self.ratio)
        groups = starts.shape[1]
        valid = torch.arange(groups, device=x.device) < count.unsqueeze(-1)
        group_positions = positions.gather(1, starts).masked_fill(~valid, 0)
        group_sequence_ids = sequence_ids.gather(1, starts).masked_fill(~valid, -1)
        if groups == 0:
            return None, group_positions, group_sequence_ids, valid
        members = (starts.unsqueeze(-1) + torch.arange(self.ratio, device=x.device)).flatten(1)

        def take(values):  # [B, groups * ratio, D] rows of the group members
            return values.gather(1, members.unsqueeze(-1).expand(-1, -1, values.shape[-1]))

        if self.gate_proj is None:
            latent = take(self.kv_proj(x))
        else:  # pooled in fp32
            batch = x.shape[0]
            kv = take(F.linear(x.float(), self.kv_proj.weight.float())).view(batch, groups, self.ratio, -1)
            gate = take(F.linear(x.float(), self.gate_proj.weight.float())).view(batch, groups, self.ratio, -1)
            latent = (kv * gate.softmax(dim=2)).sum(dim=2)
        latent = latent.masked_fill(~valid.unsqueeze(-1), 0)
        return self.norm(latent.to(x.dtype)), group_positions, group_sequence_ids, valid


@dataclass
class ShadowIndexers:
    """Global KV / index tensors shared by CSA2 layers (FULL computes, REINDEX/REUSE reuse)."""

    compressed_sequence_ids: torch.Tensor | None = None
    compressed_kv: torch.Tensor | None = None
    index_keys: torch.Tensor | None = None
    topk_indices: torch.Tensor | None = None
    candidates: torch.Tensor | None = None

    @classmethod
    def load(cls, tensors) -> "ShadowIndexers":
        return cls(*(None if t.numel() == 0 else t for t in tensors))

    def dump(self, empty: torch.Tensor) -> tuple[torch.Tensor, ...]:
        return tuple(v if v is not None else empty for v in (self.compressed_sequence_ids, self.compressed_kv,
                                                             self.index_keys, self.topk_indices, self.candidates))


def _select_topk(scores: torch.Tensor, count: int, *, stable: bool, sorted: bool = False):
    if stable:
        idx = torch.argsort(scores, dim=-1, descending=True, stable=True)[..., :count]
        return scores.gather(-1, idx), idx
    return scores.topk(count, dim=-1, sorted=sorted)


def select_candidate_blocks(scores, visible, topk_blocks, block_size, *, stable=False):
    width = scores.shape[-1]
    if width == 0:
        return torch.zeros_like(scores, dtype=torch.bool)
    blocks = F.pad(scores, (0, -width % block_size), value=float("-inf")).unflatten(-1, (-1, block_size)).amax(-1)
    last = (visible - 1) // block_size
    ids = torch.arange(blocks.shape[-1], device=scores.device)
    blocks = blocks.masked_fill(ids == last.unsqueeze(-1), torch.inf)
    values, idx = _select_topk(blocks, min(topk_blocks, blocks.shape[-1]), stable=stable, sorted=True)
    keep = torch.zeros_like(blocks, dtype=torch.bool)
    keep.scatter_(-1, idx, values > float("-inf"))
    return keep.repeat_interleave(block_size, dim=-1)[..., :width]


def visible_key_ranges(key_sequence_ids: torch.Tensor, query_sequence_ids: torch.Tensor, positions: torch.Tensor,
                       ratio: int):
    """Per query, the compressed keys it may see: ``[start, end)`` in the key axis (keys are sorted
    by sequence; a query sees its own sequence's keys whose groups ended at or before it), the
    width of the widest sequence (a host integer: it shapes the score tensor) and validity."""
    sentinel = torch.iinfo(key_sequence_ids.dtype).max
    searchable = key_sequence_ids.masked_fill(key_sequence_ids < 0, sentinel).contiguous()
    queries = query_sequence_ids.contiguous()
    first = torch.searchsorted(searchable, queries, right=False)
    past = torch.searchsorted(searchable, queries, right=True)
    end = torch.minimum(past, first + (positions + 1) // ratio)
    valid = (query_sequence_ids >= 0) & (first < end)
    return first, torch.where(valid, end, first), int((past - first).max().item())


class SparseIndexer(nn.Module):
    """Scores the compressed keys for every query (relu(q . k) weighted per head) and keeps the
    top-k. A layer that owns keys projects them from this layer's latents; the candidate-source
    layer also keeps the best key blocks, which later layers restrict their scores to."""

    def __init__(self, config: DeepSeekV41Config, layer_id: int, rotary: RotaryEmbedding) -> None:
        super().__init__()
        source = config.candidate_source_layer_id
        self.owns_keys = layer_id in config.kv_source_layer_ids
        self.is_candidate_source = layer_id == source
        self.uses_candidates = 0 <= source < layer_id
        self.ratio = config.compress_ratios[layer_id]
        self.rotary = rotary
        self.stable_topk = False  # set by callers that need ties broken by index (parity runs)
        self.quantized_cache = config.cache_quantization == "hf"
        self.num_heads, self.head_dim, self.topk = config.index_n_heads, config.index_head_dim, config.index_topk
        self.topk_blocks, self.block_size = config.candidate_topk_blocks, config.candidate_block_size
        # parameter names are the checkpoint's
        self.q_proj = Linear(config.q_lora_rank, self.num_heads * self.head_dim, bias=False)
        self.weight_proj = Linear(config.hidden_size, self.num_heads, bias=False)
        if self.owns_keys:
            self.k_proj = Linear(config.head_dim, self.head_dim, bias=False)
            self.k_norm = RMSNorm(self.head_dim, config.rms_norm_eps)

    def _fp4(self, t: torch.Tensor) -> torch.Tensor:
        return quantize_activation(t, "fp4_index") if self.quantized_cache else t

    def _refresh_keys(self, latent, group_positions, shadow: ShadowIndexers) -> None:
        shadow.index_keys = None
        if latent is not None:
            keys = apply_rope(self.k_norm(self.k_proj(latent)), group_positions, self.rotary.freqs(True))
            shadow.index_keys = self._fp4(keys).unsqueeze(1)

    def forward(self, x, q_residual, latent, group_positions, context: ModelContext, shadow: ShadowIndexers):
        if self.owns_keys:
            self._refresh_keys(latent, group_positions, shadow)
        if shadow.index_keys is None:  # nothing compressed yet: no selection (and no candidates)
            shadow.topk_indices = None
            if self.is_candidate_source:
                shadow.candidates = None
            return
        batch, length, _ = x.shape
        first, end, width = visible_key_ranges(shadow.compressed_sequence_ids, context.sequence_ids,
                                               context.positions, self.ratio)
        query = self.q_proj(q_residual).view(batch, length, self.num_heads, self.head_dim)
        query = self._fp4(apply_rope(query, context.positions, self.rotary.freqs(True)))
        head_weights = self.weight_proj(x).float() * self.num_heads ** -0.5
        scores = index_scores(query, shadow.index_keys[:, 0], head_weights, first, end, width,
                              shadow.candidates if self.uses_candidates else None)
        if self.is_candidate_source:
            shadow.candidates = select_candidate_blocks(scores, end - first, self.topk_blocks, self.block_size,
                                                        stable=self.stable_topk)
        values, idx = _select_topk(scores, min(self.topk, scores.shape[-1]), stable=self.stable_topk,
                                   sorted=self.quantized_cache)
        picked = first.unsqueeze(-1) + idx
        shadow.topk_indices = torch.where(values > float("-inf"), picked, torch.full_like(picked, -1))


class CSA2Attention(nn.Module):
    def __init__(self, config: DeepSeekV41Config, layer_id: int, rotary: RotaryEmbedding) -> None:
        super().__init__()
        self.config = config
        self.layer_id = layer_id
        self.ratio = config.compress_ratios[layer_id]
        self.num_heads = config.num_attention_heads
        self.head_dim = config.head_dim
        self.dropout = config.attention_dropout
        self.ordered_kv_grad = False
        self.rotary = rotary
        self.q_a = Linear(config.hidden_size, config.q_lora_rank, bias=False)
        self.q_norm = RMSNorm(config.q_lora_rank, config.rms_norm_eps)
        self.q_b = Linear(config.q_lora_rank, self.num_heads * self.head_dim, bias=False)
        self.kv_proj = Linear(config.hidden_size, self.head_dim, bias=False)
        self.kv_norm = RMSNorm(self.head_dim, config.rms_norm_eps)
        group_input = self.num_heads * self.head_dim // config.o_groups
        self.o_a = GroupedLinear(group_input, config.o_lora_rank, config.o_groups)
        self.o_b = Linear(config.o_groups * config.o_lora_rank, config.hidden_size, bias=False)
        self.sinks = AttentionSinks(self.num_heads)
        self.compressor = Compressor(config, layer_id) if layer_id in config.kv_source_layer_ids else None
        self.indexer = SparseIndexer(config, layer_id, rotary) if layer_id in config.index_source_layer_ids else None
        self.mode = (None if self.ratio <= 0 else CSA2Mode.FULL if self.compressor is not None
                     else CSA2Mode.REINDEX if self.indexer is not None else CSA2Mode.REUSE)

    def forward(self, x: torch.Tensor, context: ModelContext, shadow: ShadowIndexers) -> torch.Tensor:
        batch, length, _ = x.shape
        compressed = self.ratio > 0
        freqs = self.rotary.freqs(compressed)
        q_residual = self.q_norm(self.q_a(x))
        query = self.q_b(q_residual).view(batch, length, self.num_heads, self.head_dim)
        query = apply_rope(query, context.positions, freqs).transpose(1, 2)
        kv = apply_rope(self.kv_norm(self.kv_proj(x)), context.positions, freqs).unsqueeze(1)
        if self.config.cache_quantization == "hf":
            kv = quantize_activation(kv, "fp8")
        kv = context.gather_attention(kv, dim=2)[:, 0]
        entries = topk = None
        if compressed:
            latent = None
            group_positions = context.positions[:, :0]
            if self.compressor is not None:
                latent, group_positions, group_seq, _ = self.compressor(
                    context.gather(x), context.gather(context.positions), context.gather(context.token_mask),
                    context.gather(context.sequence_ids))
                shadow.compressed_sequence_ids = group_seq
                shadow.compressed_kv = shadow.index_keys = shadow.topk_indices = shadow.candidates = None
            if self.indexer is not None:
                with torch.no_grad():
                    self.indexer(x, q_residual, latent, group_positions, context, shadow)
            if latent is not None:
                rotated = apply_rope(latent, group_positions, self.rotary.freqs(True))
                if self.config.cache_quantization == "hf":
                    rotated = quantize_activation(rotated, "fp4_kv")
                shadow.compressed_kv = rotated.unsqueeze(1)
            if shadow.compressed_kv is not None and shadow.topk_indices is not None:
                entries = shadow.compressed_kv[:, 0]
                topk = shadow.topk_indices
        out = sparse_attention(query, kv, context.attention_indices, context.attention_mask[:, 0], entries, topk,
                               self.sinks(query), dropout=self.dropout if self.training else 0.0,
                               deterministic=self.ordered_kv_grad)
        out = apply_rope(out, context.positions, freqs, inverse=True)
        grouped = out.reshape(batch, length, self.config.o_groups, -1)
        return self.o_b(self.o_a(grouped).flatten(2))


__all__ = ["AttentionSinks", "CSA2Attention", "CSA2Mode", "Compressor", "GroupedLinear", "RMSNorm",
           "RotaryEmbedding", "ShadowIndexers", "SparseIndexer", "apply_rope", "complete_group_starts",
           "select_candidate_blocks", "visible_key_ranges"]
