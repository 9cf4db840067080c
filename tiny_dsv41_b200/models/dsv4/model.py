"""DeepSeek-V4.1 decoder for training: mHC residual streams, CSA2 attention, sparse MoE and
Engram n-gram memory.

Structure and parameter names follow ``dsv41_train/models/dsv4/model.py`` so released checkpoints
and native state dicts load unchanged:

* ``model.embedding``, ``model.layers.N.{attention, moe, input_norm, post_attention_norm,
  attention_hc, moe_hc, engram}``, ``model.norm``, ``model.engram_tables.<layer>``, ``lm_head``.
* Four streams per token; every branch collapses the streams with the *previous* HC's ``pre``
  weights and expands its output back with (post, comb) - ``DecoderLayer`` below.
* Engram: per-layer n-gram hash rows (``NgramHash``) gathered from row-sharded (or CPU-offloaded)
  tables, gated per stream by a signed-sqrt sigmoid of an RMS-scaled dot product.
* The load-balancing loss gradient reaches the router logits through the router's auxiliary
  gradient (no retained graph), and the LM head supports selected-token log-probabilities for RL.
"""

from __future__ import annotations

import math
from contextlib import nullcontext
from dataclasses import dataclass, fields, replace
from functools import partial
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from ... import ops
from ...ops.router import AuxGradient
from ...parallel import replay
from ...parallel.cp import ContextParallel, ModelContext
from ...parallel.dispatch import TokenDispatcher
from ...parallel.engram_offload import CPUEmbeddingLookup
from ...utils.trace import nvtx_range
from ..common import Linear, LMHead
from .attention import AttentionSinks, CSA2Attention, GroupedLinear, RMSNorm, RotaryEmbedding, ShadowIndexers
from .config import DeepSeekV41Config
from .mhc import HyperConnection
from .moe import RoutedExperts, SparseMoE, TopKRouter


def _direct(function, *args, **_kwargs):
    return function(*args)


class _ScaleGradient(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, scale):
        ctx.scale = scale
        return tensor.view_as(tensor)

    @staticmethod
    def backward(ctx, grad):
        return grad * ctx.scale, None


@dataclass
class _RowRoute:
    """Where the looked-up ids of one rank go: ``order`` groups the flat ids by owning rank
    (stable), ``send[r]`` ids are asked of rank r and ``recv[r]`` ids are asked of this rank by r."""

    order: torch.Tensor
    send: list[int]
    recv: list[int]
    group: object

    @classmethod
    def plan(cls, owners: torch.Tensor, size: int, group) -> "_RowRoute":
        asked = torch.bincount(owners, minlength=size)
        asked_of_me = torch.empty_like(asked)
        dist.all_to_all_single(asked_of_me, asked, group=group)
        return cls(torch.argsort(owners, stable=True), asked.tolist(), asked_of_me.tolist(), group)

    def requests_for_me(self, flat: torch.Tensor) -> torch.Tensor:
        incoming = flat.new_empty(sum(self.recv))
        dist.all_to_all_single(incoming, flat.index_select(0, self.order).contiguous(), output_split_sizes=self.recv,
                               input_split_sizes=self.send, group=self.group)
        return incoming

    def rows_back(self, served: torch.Tensor) -> torch.Tensor:
        import torch.distributed.nn.functional as dist_nn

        grouped = served.new_empty((sum(self.send), served.shape[1]))
        grouped = dist_nn.all_to_all_single(grouped, served.contiguous(), output_split_sizes=self.send,
                                            input_split_sizes=self.recv, group=self.group)
        # undo the grouping by owner: row k of `grouped` belongs at flat position order[k]
        return grouped.new_zeros(grouped.shape).index_copy(0, self.order, grouped)


class RowShardedEmbedding(nn.Module):
    """Embedding rows sharded over a mesh; lookups are routed to their owning rank and back.

    Owner of row r: the first ``remainder`` ranks own ``base + 1`` rows, the rest ``base`` rows
    (``dsv41_train/models/dsv4/model.py:59-178``). With ``engram_offload`` the local rows stay
    in host memory and are served by :class:`CPUEmbeddingLookup`.
    """

    def __init__(self, num_embeddings: int, embedding_dim: int, mesh=None, sparse_gradients: bool = False, *,
                 engram_offload: bool = False) -> None:
        super().__init__()
        if mesh is not None and mesh.ndim != 1:
            raise ValueError("the embedding mesh must be one-dimensional")
        if engram_offload and not sparse_gradients:
            raise ValueError("CPU Engram offload requires sparse gradients")
        self.global_num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.mesh = mesh
        self.sparse_gradients = sparse_gradients
        self.engram_offload = engram_offload
        self._cpu_lookup = CPUEmbeddingLookup() if engram_offload else None
        self.size = 1 if mesh is None else mesh.size()
        self.rank = 0 if mesh is None else mesh.get_local_rank()
        self.group = None if mesh is None else mesh.get_group()
        if num_embeddings < self.size:
            raise ValueError("embedding rows must be at least the embedding mesh size")
        base, rem = divmod(num_embeddings, self.size)
        self.row_start = self.rank * base + min(self.rank, rem)
        self.row_stop = self.row_start + base + int(self.rank < rem)
        device = torch.empty(0).device
        if engram_offload and device.type != "meta":
            device = torch.device("cpu")
        self.weight = nn.Parameter(torch.empty(self.row_stop - self.row_start, embedding_dim, device=device))

    def owners(self, flat: torch.Tensor) -> torch.Tensor:
        base, rem = divmod(self.global_num_embeddings, self.size)
        large = (base + 1) * rem
        return torch.where(flat < large, torch.div(flat, base + 1, rounding_mode="floor"),
                           rem + torch.div(flat - large, max(base, 1), rounding_mode="floor"))

    def forward(self, indices: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return self._lookup(indices)
        flat = indices.reshape(-1)
        route = _RowRoute.plan(self.owners(flat), self.size, self.group)
        wanted = route.requests_for_me(flat)
        # every owner's rows flow back to each requester; the gradient of a row that several ranks
        # requested is summed over them, so it is scaled by 1 / mesh size as the reference does
        served = _ScaleGradient.apply(self._lookup(wanted - self.row_start), 1.0 / self.size)
        return route.rows_back(served).view(*indices.shape, self.embedding_dim)

    def _lookup(self, indices: torch.Tensor) -> torch.Tensor:
        if self._cpu_lookup is not None:
            return self._cpu_lookup(self.weight, indices, device=indices.device)
        return F.embedding(indices, self.weight, sparse=self.sparse_gradients)

    def configure_cache(self, budget_bytes: int, device) -> None:
        if self._cpu_lookup is None:
            raise ValueError("Engram row caching requires CPU offload")
        self._cpu_lookup.configure_cache(budget_bytes, device)

    def clear_cache(self) -> None:
        if self._cpu_lookup is not None:
            self._cpu_lookup.clear_cache()

    def synchronize(self) -> None:
        if self._cpu_lookup is not None:
            self._cpu_lookup.synchronize()

    def _apply(self, fn, recurse=True):
        self.clear_cache()
        if self.engram_offload and not self.weight.is_meta:
            if fn(torch.empty(0, dtype=self.weight.dtype, device="cpu")).device.type != "cpu":
                raise ValueError("CPU Engram placement is explicit; load the table directly on CPU")
        return super()._apply(fn, recurse)


def _is_prime(value: int) -> bool:
    if value < 2 or value % 2 == 0:
        return value == 2
    d = 3
    while d * d <= value:
        if value % d == 0:
            return False
        d += 2
    return True


def _next_prime(value: int, used: set[int]) -> int:
    value += 1
    while value in used or not _is_prime(value):
        value += 1
    return value


def build_compressed_token_map(tokenizer_file: str | Path) -> tuple[torch.Tensor, int]:
    """Map every token id to a compressed id by its normalised text (NFKC, NFD, accent strip,
    lowercase, whitespace collapse), the table index space of the released Engram weights."""
    try:
        from tokenizers import Regex, Tokenizer, normalizers
    except ImportError as error:
        raise RuntimeError("loading Engram checkpoint weights requires the tokenizers package") from error
    tokenizer = Tokenizer.from_file(str(tokenizer_file))
    sentinel = "\ue000"
    normalizer = normalizers.Sequence([
        normalizers.NFKC(), normalizers.NFD(), normalizers.StripAccents(), normalizers.Lowercase(),
        normalizers.Replace(Regex(r"[ \t\r\n]+"), " "), normalizers.Replace(Regex(r"^ $"), sentinel),
        normalizers.Strip(), normalizers.Replace(sentinel, " "),
    ])
    compressed: dict[str, int] = {}
    mapping = []
    for token_id in range(tokenizer.get_vocab_size(with_added_tokens=True)):
        text = tokenizer.decode([token_id], skip_special_tokens=False)
        key = tokenizer.id_to_token(token_id) if "\ufffd" in text else (normalizer.normalize_str(text) or text)
        mapping.append(compressed.setdefault(key, len(compressed)))
    return torch.tensor(mapping, dtype=torch.long), len(compressed)


def _hash_multipliers(layer_ids, max_ngram: int, compressed_vocab: int) -> torch.Tensor:
    """Fixed per-layer odd multipliers (numpy PCG64 seeded with 10007 * layer) that address the
    pretrained Engram rows; they must match the checkpoint's, hence the same generator."""
    bound = max(1, (np.iinfo(np.int64).max // compressed_vocab) // 2)
    rows = []
    for layer in layer_ids:
        gen = np.random.default_rng(10007 * layer)
        rows.append(torch.from_numpy(gen.integers(0, bound, size=max_ngram, dtype=np.int64) * 2 + 1))
    return torch.stack(rows)


class NgramHash(nn.Module):
    """Rolling XOR hash of the last n compressed tokens (n = 2..max_ngram) per head, modulo a
    distinct prime per (layer, n, head), offset into the layer's table. Sequence boundaries and
    dead tokens are replaced by the pad id."""

    def __init__(self, config: DeepSeekV41Config, layer_ids=None, token_map: torch.Tensor | None = None) -> None:
        super().__init__()
        self.max_ngram = config.engram_max_ngram_size
        if token_map is None:
            token_map = torch.arange(config.vocab_size).remainder(config.engram_compressed_vocab_size)
        if token_map.ndim != 1 or token_map.shape[0] != config.vocab_size:
            raise ValueError("Engram token map must contain one entry per vocabulary id")
        if not token_map.is_meta and token_map.numel() and (
                token_map.min() < 0 or token_map.max() >= config.engram_compressed_vocab_size):
            raise ValueError("Engram token map contains an out-of-range compressed id")
        self.pad_id = (config.engram_pad_id % config.engram_compressed_vocab_size if token_map.is_meta
                       else int(token_map[config.engram_pad_id]))
        layer_ids = list(config.engram_layer_ids if layer_ids is None else layer_ids)
        if not set(layer_ids).issubset(config.engram_layer_ids):
            raise ValueError("Engram hash layers must be configured Engram layers")
        selected = set(layer_ids)
        layer_primes, layer_offsets, used = [], [], set()
        for layer, table_size in zip(config.engram_layer_ids, config.engram_num_embeddings):
            primes, offsets, offset = [], [], 0
            current = config.engram_vocab_size - 1
            for _ in range((self.max_ngram - 1) * config.engram_n_heads):
                current = _next_prime(current, used)
                used.add(current)
                primes.append(current)
                offsets.append(offset)
                offset += current
            if offset > table_size:
                raise ValueError(f"engram table needs {offset} rows, got {table_size}")
            if layer in selected:
                layer_primes.append(primes)
                layer_offsets.append(offsets)
        self.register_buffer("token_map", token_map.to(torch.long), persistent=False)
        self.register_buffer("primes", torch.tensor(layer_primes).view(len(layer_ids), self.max_ngram - 1,
                                                                        config.engram_n_heads), persistent=False)
        self.register_buffer("offsets", torch.tensor(layer_offsets), persistent=False)
        self.register_buffer("multipliers", _hash_multipliers(layer_ids, self.max_ngram,
                                                              config.engram_compressed_vocab_size), persistent=False)

    def forward(self, input_ids, token_mask, sequence_ids=None):
        if sequence_ids is None:
            sequence_ids = torch.zeros_like(input_ids)
        dead = -1
        tokens = self.token_map[input_ids].masked_fill(~token_mask, dead)
        seqs = sequence_ids.masked_fill(~token_mask, dead)
        ctx = self.max_ngram - 1
        hist = F.pad(tokens, (ctx, 0), value=dead)
        seq_hist = F.pad(seqs, (ctx, 0), value=dead)
        length = tokens.shape[1]
        shifted, blocked = [], torch.zeros_like(tokens, dtype=torch.bool)
        for distance in range(self.max_ngram):
            src = hist[:, ctx - distance: ctx - distance + length]
            src_seq = seq_hist[:, ctx - distance: ctx - distance + length]
            blocked |= (src == dead) | (src_seq != seqs)
            shifted.append(torch.where(blocked, self.pad_id, src))
        windows = torch.stack(shifted, dim=-1)
        products = windows.unsqueeze(2) * self.multipliers
        rolling, hashes = products[..., 0], []
        for n in range(1, self.max_ngram):
            rolling = torch.bitwise_xor(rolling, products[..., n])
            hashes.append(rolling.unsqueeze(-1) % self.primes[:, n - 1])
        return torch.cat(hashes, dim=-1) + self.offsets


class Engram(nn.Module):
    def __init__(self, config: DeepSeekV41Config) -> None:
        super().__init__()
        columns = (config.engram_max_ngram_size - 1) * config.engram_n_heads
        self.hidden_size = config.hidden_size
        self.hc_mult = config.hc_mult
        self.eps = config.rms_norm_eps
        self.proj = Linear(columns * config.engram_head_dim, config.hidden_size * (config.hc_mult + 1), bias=False)
        self.q_weight = nn.Parameter(torch.ones(config.hc_mult, config.hidden_size))
        self.k_weight = nn.Parameter(torch.ones(config.hc_mult, config.hidden_size))

    def forward(self, streams, rows, mask):
        key, value = self.proj(rows.flatten(-2).to(streams.dtype)).split(
            [self.hc_mult * self.hidden_size, self.hidden_size], dim=-1)
        key = key.float().unflatten(-1, (self.hc_mult, self.hidden_size))
        hidden = streams.float()
        scale = torch.rsqrt(hidden.square().mean(-1) + self.eps) * torch.rsqrt(key.square().mean(-1) + self.eps)
        dot = (hidden * self.q_weight.float() * self.k_weight.float() * key).sum(-1) * scale * self.hidden_size ** -0.5
        gate = torch.sigmoid(torch.copysign(dot.abs().clamp_min(1e-6).sqrt(), dot))
        gate = gate.masked_fill(~mask.unsqueeze(-1), 0)
        return (hidden + gate.unsqueeze(-1) * value.float().unsqueeze(-2)).to(streams.dtype)


class DecoderLayer(nn.Module):
    def __init__(self, config, layer_id, rotary, token_dispatcher) -> None:
        super().__init__()
        self.layer_id = layer_id
        self.attention = CSA2Attention(config, layer_id, rotary)
        self.moe = SparseMoE(config, token_dispatcher)
        self.input_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.engram = Engram(config) if layer_id in config.engram_layer_ids else None
        self.attention_hc = HyperConnection(config)
        self.moe_hc = HyperConnection(config)

    @staticmethod
    def _branch(hc, streams, pre_mix, body):
        """One hyper-connected branch: collapse the streams with ``pre_mix``, run ``body`` on the
        collapsed row, expand its output back into the streams; returns the new streams, the
        next branch's pre-mix weights and whatever else ``body`` returned."""
        collapsed, next_pre, post, comb = hc(streams, pre_mix)
        value, *extra = body(collapsed)
        return hc.finish(value, streams, post, comb), next_pre, extra

    def forward(self, streams, pre_mix, context, shadow, engram_rows):
        if self.engram is not None:
            streams = self.engram(streams, engram_rows, context.token_mask)
        with nvtx_range("attention"):
            streams, pre_mix, _ = self._branch(
                self.attention_hc, streams, pre_mix, lambda x: (self.attention(self.input_norm(x), context, shadow),))
        with nvtx_range("moe"):
            streams, pre_mix, (logits,) = self._branch(self.moe_hc, streams, pre_mix,
                                                       lambda x: self.moe(self.post_attention_norm(x)))
        return streams, pre_mix, logits


class DeepSeekV41Model(nn.Module):
    def __init__(self, config, context_parallel=None, token_dispatcher=None, engram_mesh=None, layer_ids=None,
                 sparse_engram_gradients=False, engram_offload=False) -> None:
        super().__init__()
        self.config = config
        self.context_parallel = context_parallel or ContextParallel()
        token_dispatcher = token_dispatcher or TokenDispatcher()
        layer_ids = list(range(config.num_hidden_layers)) if layer_ids is None else list(layer_ids)
        if not layer_ids or any(not 0 <= i < config.num_hidden_layers for i in layer_ids):
            raise ValueError("layer_ids must select at least one configured layer")
        self.layer_ids = layer_ids
        self.embedding = nn.Embedding(config.vocab_size, config.hidden_size)
        self.rotary = RotaryEmbedding(config)
        self.layers = nn.ModuleList(DecoderLayer(config, i, self.rotary, token_dispatcher) for i in layer_ids)
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        sizes = dict(zip(config.engram_layer_ids, config.engram_num_embeddings))
        self.engram_layer_ids = [i for i in config.engram_layer_ids if i in layer_ids]
        self.hash = NgramHash(config, self.engram_layer_ids) if self.engram_layer_ids else None
        self.engram_tables = nn.ModuleDict({
            str(i): RowShardedEmbedding(sizes[i], config.engram_head_dim, engram_mesh,
                                        sparse_gradients=sparse_engram_gradients, engram_offload=engram_offload)
            for i in self.engram_layer_ids})
        self.gradient_checkpointing = False

    def _inputs(self, input_ids, attention_mask, sequence_ids):
        """Validated (ids, live-token mask, sequence ids with padding set to -1) on the embedding's
        device."""
        if input_ids.ndim != 2 or input_ids.shape[1] == 0:
            raise ValueError("input_ids must have shape [batch, nonempty sequence]")
        input_ids = input_ids.to(self.embedding.weight.device)
        if input_ids.shape[1] > self.config.max_position_embeddings:
            raise ValueError("sequence is longer than max_position_embeddings")
        for name, given in (("attention_mask", attention_mask), ("sequence_ids", sequence_ids)):
            if given is not None and given.shape != input_ids.shape:
                raise ValueError("attention_mask must match input_ids" if name == "attention_mask"
                                 else "sequence_ids must have the same shape as input_ids")
        live = (torch.ones_like(input_ids, dtype=torch.bool) if attention_mask is None
                else attention_mask.to(device=input_ids.device, dtype=torch.bool))
        seq = torch.zeros_like(input_ids) if sequence_ids is None else sequence_ids.to(input_ids.device)
        return input_ids, live, seq.masked_fill(~live, -1)

    def _engram_rows(self, input_ids, live, sequence_ids) -> dict:
        """Per Engram layer, the rows its n-gram hashes select (this CP rank's tokens)."""
        if self.hash is None:
            return {}
        hashes = self.context_parallel.shard(self.hash(input_ids, live, sequence_ids))
        return {layer: self.engram_tables[str(layer)](hashes[:, :, slot])
                for slot, layer in enumerate(self.engram_layer_ids)}

    def _context_on(self, contexts: dict, device):
        if device not in contexts:  # layers placed on several devices each get a copy of the context
            base = next(iter(contexts.values()))
            contexts[device] = replace(base, **{f.name: getattr(base, f.name).to(device) for f in fields(base)
                                                if isinstance(getattr(base, f.name), torch.Tensor)})
        return contexts[device]

    def forward(self, input_ids, attention_mask=None, sequence_ids=None):
        input_ids, live, sequence_ids = self._inputs(input_ids, attention_mask, sequence_ids)
        context = ModelContext.build(self.context_parallel, input_ids, live, sequence_ids, self.config.sliding_window)
        contexts = {input_ids.device: context}
        engram_rows = self._engram_rows(input_ids, live, sequence_ids)
        hidden = self.embedding(context.input_ids)
        # hc_mult copies of the embedding; the first branch collapses them with weight 1 on stream 0
        streams = hidden.unsqueeze(2).repeat(1, 1, self.config.hc_mult, 1)
        pre_mix = torch.nn.functional.one_hot(torch.zeros(hidden.shape[:2], dtype=torch.long, device=hidden.device),
                                              self.config.hc_mult).float()
        none = hidden.new_empty(0)
        shadow = ShadowIndexers().dump(none)
        checkpointed = self.gradient_checkpointing and self.training and torch.is_grad_enabled()
        run = partial(checkpoint, context_fn=replay.checkpoint_contexts) if checkpointed else _direct
        router_logits = []
        for layer in self.layers:
            device = next(layer.parameters()).device
            local = self._context_on(contexts, device)
            streams, pre_mix = streams.to(device), pre_mix.to(device)
            step = lambda *args, current=layer, ctx=local: self._forward_layer(current, ctx, *args)  # noqa: E731
            streams, pre_mix, logits, *shadow = run(step, streams, pre_mix,
                                                    engram_rows.get(layer.layer_id, none).to(device),
                                                    *(t.to(device) for t in shadow), use_reentrant=False)
            router_logits.append(logits)
        device = self.norm.weight.device
        with torch.cuda.device(device) if device.type == "cuda" else nullcontext():
            return self.norm(HyperConnection.collapse(streams.to(device), pre_mix.to(device))), tuple(router_logits)

    def _forward_layer(self, layer, context, streams, pre_mix, engram_row, *shadow_tensors):
        shadow = ShadowIndexers.load(shadow_tensors)
        with torch.cuda.device(streams.device) if streams.is_cuda else nullcontext():
            streams, pre_mix, logits = layer(streams, pre_mix, context, shadow,
                                             None if engram_row.numel() == 0 else engram_row)
        return streams, pre_mix, logits, *shadow.dump(streams.new_empty(0))


def load_balancing_loss(router_logits, num_experts: int, topk: int, attention_mask, context_parallel=None):
    """E * sum_e f_e * P_e over the live tokens of all layers: f_e is the fraction of top-k
    assignments that go to expert e, P_e the mean router probability of e (softmax of the fp32
    logits); under context parallelism both are totalled over the CP group first."""
    device = router_logits[0].device
    probs = torch.softmax(torch.cat([logits.float().to(device) for logits in router_logits]), dim=-1)
    layers = len(router_logits)
    if attention_mask is None:
        weight = torch.ones(probs.shape[0], device=device)
    else:
        weight = attention_mask.flatten().float().to(device).repeat(layers)
    chosen = probs.topk(topk, dim=-1).indices
    counts = torch.zeros(num_experts, device=device).index_add(0, chosen.flatten(), weight.repeat_interleave(topk))
    mass = (probs * weight.unsqueeze(-1)).sum(0)
    tokens = weight.sum()
    if context_parallel is not None:
        counts = context_parallel.sum(counts)
        mass = context_parallel.sum(mass, autograd=True)
        tokens = context_parallel.sum(tokens)
    return num_experts * ((counts / tokens) * (mass / tokens)).sum()


@dataclass
class CausalLMOutput:
    loss: torch.Tensor | None
    logits: torch.Tensor | None
    aux_loss: torch.Tensor | None
    router_logits: tuple[torch.Tensor, ...]
    token_log_probs: torch.Tensor | None = None


class DeepSeekV41ForCausalLM(nn.Module):
    def __init__(self, config, context_parallel=None, token_dispatcher=None, engram_mesh=None, layer_ids=None,
                 sparse_engram_gradients=False, engram_offload=False) -> None:
        super().__init__()
        self.config = config
        self.context_parallel = context_parallel or ContextParallel()
        self.model = DeepSeekV41Model(config, self.context_parallel, token_dispatcher, engram_mesh, layer_ids,
                                      sparse_engram_gradients, engram_offload)
        self.lm_head = LMHead(config.hidden_size, config.vocab_size)
        self.aux_gradient = AuxGradient()
        for module in self.modules():
            if isinstance(module, TopKRouter):
                module.aux = self.aux_gradient
        self.apply(self._initialize)

    def _initialize(self, module: nn.Module) -> None:
        if any(p.is_meta for p in module.parameters(recurse=False)):
            return
        std = self.config.initializer_range
        if isinstance(module, (nn.Linear, nn.Embedding, RowShardedEmbedding)):
            nn.init.normal_(module.weight, std=std)
        if isinstance(module, RMSNorm):
            nn.init.ones_(module.weight)
        elif isinstance(module, HyperConnection):
            nn.init.normal_(module.fn, std=std)
            nn.init.zeros_(module.base)
            nn.init.ones_(module.scale)
        elif isinstance(module, GroupedLinear):
            nn.init.normal_(module.weight, std=std)
        elif isinstance(module, TopKRouter):
            nn.init.normal_(module.weight, std=std)
            nn.init.zeros_(module.selection_bias)
        elif isinstance(module, RoutedExperts):
            if module.gate_up.is_meta:
                return
            if module.num_experts == module.global_num_experts:
                nn.init.normal_(module.gate_up, std=std)
                nn.init.normal_(module.down, std=std)
            else:
                gen = torch.Generator(device=module.gate_up.device)
                gen.manual_seed(torch.initial_seed() + module.expert_start)
                nn.init.normal_(module.gate_up, std=std, generator=gen)
                nn.init.normal_(module.down, std=std, generator=gen)

    def gradient_checkpointing_enable(self) -> None:
        self.model.gradient_checkpointing = True

    def _token_log_probs(self, hidden, targets, mask, temperature):
        selected = self.lm_head(hidden[mask], targets[mask], mode="logprob", temperature=temperature)
        return selected.new_zeros(mask.shape).masked_scatter(mask, selected)

    def fp32_island_parameters(self):
        """mHC mixing parameters and attention sinks stay fp32 under bf16 training."""
        return [p for m in self.modules() if isinstance(m, (HyperConnection, AttentionSinks))
                for p in m.parameters(recurse=False)]

    def to_mixed_precision(self, dtype=torch.bfloat16):
        """Cast to `dtype` except the fp32 islands (and fp32 buffers such as the routing bias)."""
        islands = {id(p) for p in self.fp32_island_parameters()}
        for module in self.modules():
            for name, param in list(module.named_parameters(recurse=False)):
                if id(param) not in islands and param.is_floating_point():
                    param.data = param.data.to(dtype)
        return self

    def forward(self, input_ids, attention_mask=None, labels=None, sequence_ids=None, *, target_ids=None,
                target_mask=None, temperature: float = 1.0, compute_aux_loss: bool = True) -> CausalLMOutput:
        """With ``labels``: shifted CE mean (packed boundaries masked). With ``target_ids``: aligned
        per-token log-probabilities ([batch, local sequence], zero where masked)."""
        token_mask = (torch.ones_like(input_ids, dtype=torch.bool) if attention_mask is None
                      else attention_mask.to(device=input_ids.device, dtype=torch.bool))
        if token_mask.shape != input_ids.shape:
            raise ValueError("attention_mask must match input_ids")
        if target_ids is None and target_mask is not None:
            raise ValueError("target_mask requires target_ids")
        if target_ids is not None:
            if labels is not None:
                raise ValueError("labels and target_ids are mutually exclusive")
            if target_ids.shape != input_ids.shape or target_ids.dtype != torch.long:
                raise ValueError("target_ids must be int64 with the same shape as input_ids")
            if not math.isfinite(temperature) or temperature <= 0:
                raise ValueError("temperature must be finite and positive")
            if target_mask is not None and target_mask.shape != input_ids.shape:
                raise ValueError("target_mask must match input_ids")
            target_mask = token_mask if target_mask is None else (
                target_mask.to(device=input_ids.device, dtype=torch.bool) & token_mask)
            target_ids = target_ids.to(input_ids.device)
            chosen = target_ids[target_mask]
            if ((chosen < 0) | (chosen >= self.config.vocab_size)).any():
                raise ValueError("target token ID is outside the model vocabulary")
        self.aux_gradient.set(None)
        hidden, router_logits = self.model(input_ids, token_mask, sequence_ids)
        cp = self.context_parallel
        logits = loss = token_log_probs = None
        if target_ids is not None:
            targets = cp.shard(target_ids).to(hidden.device)
            mask = cp.shard(target_mask).to(hidden.device)
            loader = checkpoint if self.training and torch.is_grad_enabled() else _direct
            token_log_probs = loader(self._token_log_probs, hidden, targets, mask, temperature, use_reentrant=False)
        elif labels is not None:
            labels = labels.to(input_ids.device)
            targets = torch.full_like(labels, -100)
            targets[:, :-1] = labels[:, 1:]
            targets[:, :-1].masked_fill_(~token_mask[:, 1:], -100)
            if sequence_ids is not None:
                targets[:, :-1].masked_fill_(sequence_ids[:, :-1] != sequence_ids[:, 1:], -100)
            targets = cp.shard(targets).to(hidden.device)
            loss_sum = self.lm_head(hidden, targets, mode="ce_sum")
            loss = cp.mean_loss(loss_sum, (targets != -100).sum())
        else:
            logits = self.lm_head(hidden)
        if not compute_aux_loss:
            return CausalLMOutput(loss, logits, None, router_logits, token_log_probs)
        local_mask = cp.shard(token_mask)
        with torch.no_grad():
            aux_loss = load_balancing_loss(tuple(l.detach() for l in router_logits), self.config.n_routed_experts,
                                           self.config.num_experts_per_tok, local_mask, None)
        coefficient = self.config.router_aux_loss_coef
        if loss is not None and torch.is_grad_enabled() and coefficient:
            self._stage_aux_gradient(router_logits, local_mask, coefficient)
        if loss is not None:
            loss = loss + coefficient * aux_loss.detach().to(loss.device)
        return CausalLMOutput(loss, logits, aux_loss, router_logits, token_log_probs)

    @torch.no_grad()
    def _stage_aux_gradient(self, router_logits, mask, coefficient):
        """d(coef * aux)/d softmax(logits) = coef * E * assignments_e / total^2 (times the token mask)."""
        experts, topk = self.config.n_routed_experts, self.config.num_experts_per_tok
        cp = self.context_parallel
        device = router_logits[0].device
        m = mask.flatten().float().to(device)
        assignments = torch.zeros(experts, device=device)
        total = torch.zeros((), device=device)
        for logits in router_logits:
            selected = torch.softmax(logits.float(), dim=-1).topk(topk, dim=-1).indices
            assignments.scatter_add_(0, selected.flatten(), m.repeat_interleave(topk))
            total += m.sum()
        assignments, total = cp.sum(assignments), cp.sum(total)
        vector = coefficient * experts * assignments / (total * total)
        self.aux_gradient.set(vector, None if bool(m.min() > 0) else m)


DeepseekV41ForCausalLM = DeepSeekV41ForCausalLM

__all__ = ["CausalLMOutput", "DeepSeekV41Config", "DeepSeekV41ForCausalLM", "DeepSeekV41Model",
           "DeepseekV41ForCausalLM", "Engram", "NgramHash", "RowShardedEmbedding", "build_compressed_token_map",
           "load_balancing_loss"]
