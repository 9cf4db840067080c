"""Snapshot the live query adapters of a DeepSeek-V4.1 learner as a vLLM LoRA update packet
(``dsv41_train/rl/lora_export.py:26-138``).

Adapters must be this library's unmerged ``LoRALinear`` on ``model.layers.N.attention.q_a`` for
exactly the configured layers, bf16, rank/alpha of the profile, dropout 0; every base parameter
must be frozen with no gradient; an optimizer, if given, must hold exactly the adapters with
finite state. Names become ``language_model.model.layers.N.attn.wq_a.lora_{A,B}.weight`` (A:
[rank, hidden], B: [q_lora_rank, rank]) and the tensors are packed with
``rollout.lora_transport.pack_update`` (peft ``{r, lora_alpha, target_modules: ["wq_a"]}``).

Under FSDP every rank calls at the same point: ranks first agree on validation status and
inventory (so one rank's failure cannot strand the others inside a gather), then sharded
adapters are gathered; rank 0 returns ``(manifest, payload)``, others ``None``.
"""

from __future__ import annotations

import re

import torch
import torch.distributed as dist

from ..rollout.lora_transport import pack_update
from .lora_config import DistributedLoRAConfig

_MODULE = re.compile(r"model\.layers\.(\d+)\.attention\.q_a\Z")
_SHA = re.compile(r"[0-9a-f]{64}\Z")


def text_dimensions(config) -> tuple[int, int, int, int]:
    """(hidden, q_lora_rank, head_dim, layers) of a config object or mapping (``text_config`` aware)."""
    def get(obj, name):
        return obj[name] if isinstance(obj, dict) else getattr(obj, name)

    try:
        nested = get(config, "text_config")
    except (AttributeError, KeyError):
        nested = None
    cfg = nested or config
    values = tuple(int(get(cfg, n)) for n in ("hidden_size", "q_lora_rank", "head_dim", "num_hidden_layers"))
    if any(v <= 0 for v in values):
        raise ValueError("DeepSeek text dimensions must be positive")
    return values


def _select(model, optimizer, profile: DistributedLoRAConfig) -> dict:
    from ..lora import LoRALinear

    hidden, q_rank, _, layers = text_dimensions(model.config)
    wanted = set(profile.selected_layers(layers))
    found, selected = set(), {}
    for name, module in sorted(model.named_modules()):
        if not (hasattr(module, "lora_a") or hasattr(module, "lora_b")):
            continue
        match = _MODULE.fullmatch(name)
        cfg = getattr(module, "config", None)
        ok = (match is not None and int(match[1]) in wanted and isinstance(module, LoRALinear)
              and getattr(cfg, "rank", None) == profile.rank and getattr(cfg, "alpha", None) == profile.alpha
              and getattr(cfg, "dropout", None) == 0 and module.scaling == profile.alpha / profile.rank
              and module.adapters_enabled and not module.merged)
        if not ok:
            raise ValueError("export requires unmerged query-only adapters matching the configured profile")
        layer = int(match[1])
        found.add(layer)
        prefix = f"language_model.model.layers.{layer}.attn.wq_a"
        for attr, letter, shape in (("lora_a", "A", (profile.rank, hidden)), ("lora_b", "B", (q_rank, profile.rank))):
            p = getattr(module, attr)
            if not p.requires_grad or p.dtype != torch.bfloat16 or tuple(p.shape) != shape:
                raise ValueError("query adapter parameter shape, dtype, or trainable flag differs")
            if hasattr(p, "device_mesh") and (not dist.is_initialized() or p.device_mesh.size() != dist.get_world_size()):
                raise ValueError("adapter DTensor mesh must span the whole export world")
            if p.grad is not None:
                g = p.grad.to_local() if hasattr(p.grad, "to_local") else p.grad
                if not bool(torch.isfinite(g).all()):
                    raise ValueError("adapter gradient is nonfinite")
            selected[f"{prefix}.lora_{letter}.weight"] = p
    if found != wanted:
        raise ValueError("query adapter inventory does not cover every configured layer")
    ids = {id(p) for p in selected.values()}
    if any(p.requires_grad or p.grad is not None for p in model.parameters() if id(p) not in ids):
        raise ValueError("all base parameters must remain frozen and have no gradients")
    if optimizer is not None:
        optimized = [p for g in optimizer.param_groups for p in g["params"]]
        if len(optimized) != len(ids) or {id(p) for p in optimized} != ids:
            raise ValueError("optimizer must contain every adapter exactly once and no base parameter")
        for state in optimizer.state.values():
            for v in state.values():
                if isinstance(v, torch.Tensor):
                    v = v.to_local() if hasattr(v, "to_local") else v
                    if not bool(torch.isfinite(v).all()):
                        raise ValueError("optimizer state is nonfinite")
    return selected


@torch.no_grad()
def export_q_a_update(model, *, version: int, lineage: str, adapter_id: int, base_identity: dict, optimizer=None,
                      lora_config: DistributedLoRAConfig | None = None):
    profile = lora_config or getattr(model, "distributed_lora_config", DistributedLoRAConfig())
    error, selected, signature = None, {}, []
    try:
        if not isinstance(profile, DistributedLoRAConfig):
            raise ValueError("export LoRA configuration must be DistributedLoRAConfig")
        if (not isinstance(base_identity, dict) or set(base_identity) != {"config_sha256", "index_sha256"}
                or any(not isinstance(v, str) or not _SHA.fullmatch(v) for v in base_identity.values())):
            raise ValueError("export requires exact mounted config/index SHA256 identity")
        selected = _select(model, optimizer, profile)
        signature = [(n, list(v.shape), str(v.dtype)) for n, v in selected.items()]
    except Exception as exc:  # agreed on below before any collective
        error = str(exc)
    if dist.is_initialized():
        status = [None] * dist.get_world_size()
        dist.all_gather_object(status, {"error": error, "signature": signature,
                                        "policy": [version, lineage, adapter_id, base_identity]})
        if any(s["error"] for s in status):
            raise ValueError("a world rank rejected adapter export validation: "
                             + "; ".join(str(s["error"]) for s in status if s["error"]))
        if any(s != status[0] for s in status):
            raise ValueError("world ranks disagree on adapter inventory or policy identity")
    elif error:
        raise ValueError(error)
    tensors = {}
    for name, p in selected.items():
        v = p.detach()
        if hasattr(v, "full_tensor"):
            v = v.full_tensor()
        tensors[name] = v.cpu().contiguous().clone()
    packet = pack_update(tensors, version=version, lineage=lineage, adapter_id=adapter_id,
                         peft={"r": profile.rank, "lora_alpha": profile.alpha, "target_modules": ["wq_a"]},
                         base_identity=base_identity)
    return packet if not dist.is_initialized() or dist.get_rank() == 0 else None


__all__ = ["export_q_a_update", "text_dimensions"]
