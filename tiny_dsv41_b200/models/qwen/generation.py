"""Incremental decoding for Qwen3-MoE: a per-request KV cache
(the native request cache of ``rollout_manager/backends/qwen_kv_cache.py:22-193``).

``KVCache`` stores each layer's post-RoPE keys and values and their positions; the attention
module appends the new tokens' entries and attends over everything cached so far (a position-based
causal mask). ``IncrementalLogits`` keeps one request's cache: called with a token sequence that
extends the cached prefix it runs only the new tokens; any other sequence restarts with a prefill.
"""

from __future__ import annotations

import torch


class KVCache:
    def __init__(self) -> None:
        self.keys: dict[int, torch.Tensor] = {}
        self.values: dict[int, torch.Tensor] = {}
        self.positions: dict[int, torch.Tensor] = {}

    def append(self, layer: int, k, v, positions):
        if layer in self.keys:
            self.keys[layer] = torch.cat((self.keys[layer], k), dim=1)
            self.values[layer] = torch.cat((self.values[layer], v), dim=1)
            self.positions[layer] = torch.cat((self.positions[layer], positions), dim=1)
        else:
            self.keys[layer], self.values[layer], self.positions[layer] = k, v, positions
        return self.keys[layer], self.values[layer], self.positions[layer]


class IncrementalLogits:
    """Next-token logits for a growing single sequence, reusing the cache across calls."""

    def __init__(self, model) -> None:
        self.model = model  # Qwen3MoeForCausalLM
        self.ids: list[int] = []
        self.cache: KVCache | None = None
        self.prefills = 0

    @torch.no_grad()
    def __call__(self, input_ids: torch.Tensor) -> torch.Tensor:
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("incremental decoding serves one sequence")
        ids = input_ids[0].tolist()
        if self.cache is None or len(ids) <= len(self.ids) or ids[:len(self.ids)] != self.ids:
            self.cache, self.ids, new = KVCache(), [], ids
            self.prefills += 1
        else:
            new = ids[len(self.ids):]
        start = len(self.ids)
        tokens = torch.tensor([new], dtype=torch.long, device=input_ids.device)
        positions = torch.arange(start, start + len(new), device=input_ids.device).unsqueeze(0)
        inner = self.model.model
        hidden = inner(tokens, None, positions, cache=self.cache).last_hidden_state
        self.ids = ids
        return self.model.lm_head(hidden[:, -1:])[:, -1]


__all__ = ["IncrementalLogits", "KVCache"]
