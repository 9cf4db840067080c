"""RL policies: a model family behind one checkpoint interface.

Behaviour of ``dsv41_train/rl/policy.py:23-483`` and ``dsv41_train/rl/qwen_policy.py:18-239``:

* A policy splits its state into *trainable* tensors (saved in every policy artifact) and
  *frozen* tensors (saved unless they can be rebuilt from the identified base: LoRA scope, or
  Qwen, whose frozen base is always the mounted checkpoint).
* Frozen base parameters are checked for identity and in-place writes (tensor ``_version``)
  before every publication, so a bug that mutates the base cannot silently leak into rollouts.
* DeepSeek-V4.1: trainable scope ``all`` or ``lora``; Engram tables are frozen and, with
  offload, stay in host memory; sparse indexers are frozen; mHC / attention-sink fp32 islands
  survive dtype casts; the model returns selected-token log-probs directly
  (``supports_token_log_probs``).
* Qwen3-MoE: scope ``all``, ``lm_head`` or ``lora``; action log-probs are replayed prefix by
  prefix, one forward per action, so the learner sees the same shapes as serial sampling.
* Layers are spread over the policy's devices with ``layer_device_map``.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch
from torch import nn

from ..lora import LoRAConfig, inject_lora, load_adapter_state, read_adapter, validate_adapter_layout
from .parallel import layer_device_map, pin_inputs_to, validate_available_devices


class _PolicyBase(nn.Module):
    trainable_scope = "all"

    def _frozen_params(self):
        return {n: p for n, p in self.named_parameters() if not p.requires_grad}

    def _capture_frozen(self) -> None:
        self._frozen = {n: (p, p._version) for n, p in self._frozen_params().items()}

    def assert_invariants(self) -> None:
        frozen = getattr(self, "_frozen", None)
        if frozen is None:
            return
        current = self._frozen_params()
        if current.keys() != frozen.keys():
            raise RuntimeError("frozen parameter set changed")
        for name, (param, version) in frozen.items():
            if current[name] is not param or param._version != version:
                raise RuntimeError(f"immutable base parameter changed: {name}")

    def requires_grad_(self, requires_grad: bool = True):
        self.assert_invariants()
        super().requires_grad_(requires_grad)
        self._capture_frozen()
        return self

    # the reference's name for the same check
    assert_engram_invariants = assert_invariants

    def frozen_parameter_fingerprint(self) -> dict:
        self.assert_invariants()
        digest = hashlib.sha256()
        for name, param in sorted(self._frozen_params().items()):
            if "norm" in name:
                digest.update(name.encode())
                digest.update(param.detach().float().cpu().numpy().tobytes())
        return {"normalization_sha256": digest.hexdigest(),
                "frozen_parameter_count": sum(p.numel() for p in self._frozen_params().values()),
                "trainable_parameter_count": sum(p.numel() for p in self.parameters() if p.requires_grad)}

    def _trainable(self):
        return {n: p for n, p in self.named_parameters() if p.requires_grad}

    def _frozen_state(self):
        return {}

    def trainable_state_dict(self) -> dict:
        self.assert_invariants()
        return {n: p.detach().cpu().clone() for n, p in self._trainable().items()}

    def frozen_state_dict(self) -> dict:
        self.assert_invariants()
        return {n: v.detach().cpu().clone() for n, v in self._frozen_state().items()}

    @torch.no_grad()
    def _load(self, state: dict, destinations: dict, what: str) -> None:
        if state.keys() != destinations.keys():
            raise ValueError(f"{what} state keys do not match the policy")
        for name, value in destinations.items():
            if tuple(value.shape) != tuple(state[name].shape):
                raise ValueError(f"{what} tensor shape mismatch: {name}")
        for name, value in destinations.items():
            value.copy_(state[name].to(device=value.device, dtype=value.dtype))

    def load_trainable_state_dict(self, state: dict) -> None:
        self.assert_invariants()
        self._load(state, self._trainable(), "trainable")

    def load_frozen_state_dict(self, state: dict) -> None:
        destinations = self._frozen_state()
        if not destinations:
            if state:
                raise ValueError("frozen weights of this policy rebuild from the identified base")
            return
        self._load(state, destinations, "frozen")
        self._capture_frozen()

    @property
    def engram_device(self) -> str:
        return "none"

    @property
    def engram_shared(self) -> bool:
        return False


class DSV41Policy(_PolicyBase):
    supports_token_log_probs = True

    def __init__(self, backend, *, trainable_scope: str = "all", engram_offload: bool = True) -> None:
        super().__init__()
        if trainable_scope not in {"all", "lora"}:
            raise ValueError("DeepSeek RL requires trainable_scope=all or lora")
        self.backend, self.config = backend, backend.config
        self.trainable_scope = trainable_scope
        self.engram_offload = engram_offload
        for table in backend.model.engram_tables.values():
            table.weight.requires_grad_(False)
        for layer in backend.model.layers:
            indexer = getattr(layer.attention, "indexer", None)
            if indexer is not None:  # frozen, with prefix-stable top-k so replay matches sampling
                indexer.stable_topk = True
                indexer.requires_grad_(False)
        if trainable_scope == "lora":
            for name, p in self.named_parameters():
                p.requires_grad_(name.endswith((".lora_a", ".lora_b")))

    @property
    def engram_device(self) -> str:
        return ",".join(sorted({str(t.weight.device) for t in self.backend.model.engram_tables.values()})) or "none"

    def _frozen_state(self):
        if self.trainable_scope == "lora":
            return {}
        state = dict(self._frozen_params())
        state.update({n: b for n, b in self.named_buffers()})
        return state

    def to_training_devices(self, devices, dtype):
        placement = layer_device_map(len(self.backend.model.layers), devices)
        validate_available_devices(devices)
        if dtype != torch.float32:
            self.backend.to_mixed_precision(dtype)
        model = self.backend.model
        tables = {id(t) for t in model.engram_tables.values()}
        model.embedding.to(placement[0])
        if model.hash is not None:
            model.hash.to(placement[0])
        for layer, device in zip(model.layers, placement):
            layer.to(device)
            table = model.engram_tables[str(layer.layer_id)] if str(layer.layer_id) in model.engram_tables else None
            if table is not None and not self.engram_offload:
                table.to(device)
        model.norm.to(placement[-1])
        self.backend.lm_head.to(placement[-1])
        del tables
        self._capture_frozen()
        return self

    def forward(self, input_ids, attention_mask=None, *, target_ids=None, target_mask=None, temperature=1.0,
                sequence_ids=None):
        out = self.backend(input_ids, attention_mask=attention_mask, sequence_ids=sequence_ids, target_ids=target_ids,
                           target_mask=target_mask, temperature=temperature, compute_aux_loss=False)
        return out.logits if target_ids is None else out.token_log_probs


LAST_POSITION_LOGITS_PATH = "last_position_head_v1"


def validate_qwen_config(config) -> None:
    if config.model_type != "qwen3_moe":
        raise ValueError("native Qwen RL requires model_type=qwen3_moe")
    if config.attention_dropout:
        raise ValueError("RL policies require attention_dropout=0")
    if config.attention_bias or config.hidden_act != "silu":
        raise ValueError("native Qwen RL requires attention_bias=false and hidden_act=silu")
    if config.rope_scaling is not None or config.use_sliding_window or config.tie_word_embeddings:
        raise ValueError("native Qwen RL does not support RoPE scaling, sliding windows or tied embeddings")


class QwenPolicy(_PolicyBase):
    def __init__(self, backend, *, trainable_scope: str = "all") -> None:
        super().__init__()
        validate_qwen_config(backend.config)
        if trainable_scope not in {"all", "lm_head", "lora"}:
            raise ValueError("Qwen trainable_scope must be all, lm_head or lora")
        self.backend, self.config = backend, backend.config
        self.trainable_scope = trainable_scope
        self.qwen_last_position_only = False
        self.qwen_kv_cache = False
        self._hooks = []
        for name, p in self.named_parameters():
            if trainable_scope == "lora":
                p.requires_grad_(name.endswith((".lora_a", ".lora_b")))
            else:
                p.requires_grad_(trainable_scope == "all" or name == "backend.lm_head.weight")
        if trainable_scope == "lora" and not any(p.requires_grad for p in self.parameters()):
            raise ValueError("inject LoRA before constructing a Qwen LoRA policy")

    def to_training_devices(self, devices, dtype):
        placement = layer_device_map(self.config.num_hidden_layers, devices)
        validate_available_devices(devices)
        self.to(dtype=dtype)
        model = self.backend.model
        for handle in self._hooks:
            handle.remove()
        model.embed_tokens.to(placement[0])
        self._hooks = [pin_inputs_to(model.embed_tokens, placement[0])]
        for layer, device in zip(model.layers, placement):
            layer.to(device)
            self._hooks.append(pin_inputs_to(layer, device))
        model.norm.to(placement[-1])
        self.backend.lm_head.to(placement[-1])
        self._hooks += [pin_inputs_to(model.norm, placement[-1]), pin_inputs_to(self.backend.lm_head, placement[-1])]
        self._capture_frozen()
        return self

    def forward(self, input_ids, attention_mask=None, *, last_position_only=False):
        if input_ids.ndim != 2 or not 0 < input_ids.shape[1] <= self.config.max_position_embeddings:
            raise ValueError("input_ids must be [batch, sequence] within max_position_embeddings")
        model = self.backend.model
        hidden = model(input_ids, attention_mask).last_hidden_state
        if last_position_only:
            hidden = hidden[:, -1:].clone()
        return self.backend.lm_head(hidden)

    def next_token_logits(self, input_ids, attention_mask=None):
        if self.qwen_kv_cache and not torch.is_grad_enabled():
            if getattr(self, "_session", None) is None:
                from ..models.qwen.generation import IncrementalLogits

                self._session = IncrementalLogits(self.backend)
            return self._session(input_ids)
        logits = self(input_ids, attention_mask, last_position_only=self.qwen_last_position_only)
        return logits[:, -1]

    def _load(self, state, destinations, what):
        self._session = None  # cached keys/values belong to the previous weights
        super()._load(state, destinations, what)

    def response_log_probs(self, prompt_ids, response_ids, temperature):
        """One forward per action over its exact sampling prefix (stop tokens included)."""
        device = next(self.parameters()).device
        values = []
        for index, token in enumerate(response_ids):
            tokens = torch.tensor([list(prompt_ids) + list(response_ids[:index])], dtype=torch.long, device=device)
            logits = self.next_token_logits(tokens, torch.ones_like(tokens))[0]
            if token >= logits.shape[-1]:
                raise ValueError("response token ID is outside the model vocabulary")
            values.append((logits.float() / temperature).log_softmax(-1)[token])
        return torch.stack(values)


def _native_dsv4_state(root: Path):
    from ..utils.safetensors_io import ShardedSafeTensorReader

    for stem in ("model.safetensors", "model.safetensors.index.json"):
        if (root / stem).is_file():
            reader = ShardedSafeTensorReader(root)
            return {name: reader.tensor(name) for name in reader.weight_map}, reader
    for stem in ("pytorch_model.bin",):
        if (root / stem).is_file():
            return torch.load(root / stem, map_location="cpu", weights_only=True), None
    raise FileNotFoundError(f"no model.safetensors or pytorch_model.bin checkpoint found in {root}")


def _adapter(model_dir, lora_config, initial_adapter, random_init):
    if lora_config is None or initial_adapter is None:
        return None
    return read_adapter(initial_adapter)


def build_dsv41_policy(model_dir, config, *, random_init: bool, devices, dtype, lora_config: LoRAConfig | None = None,
                       initial_adapter=None, engram_offload: bool = True, sft_source=None):
    from ..models.dsv4.model import DeepSeekV41ForCausalLM, NgramHash

    layer_device_map(config.num_hidden_layers, devices)
    validate_available_devices(devices)
    root = Path(model_dir)
    kwargs = dict(sparse_engram_gradients=engram_offload, engram_offload=engram_offload)
    if random_init:
        backend = DeepSeekV41ForCausalLM(config, **kwargs)
    elif getattr(config, "checkpoint_format", "native") == "released" or (root / "model.safetensors.index.json").is_file() \
            and _is_released(root):
        from ..models.dsv4.checkpoint import load_dsv41_backbone_prefix

        backend = load_dsv41_backbone_prefix(root, num_layers=config.num_hidden_layers, device="cpu",
                                             dtype=torch.float32)
    else:
        backend = DeepSeekV41ForCausalLM(config, **kwargs)
        state, reader = _native_dsv4_state(root)
        expected = backend.state_dict()
        if state.keys() != expected.keys():
            raise ValueError(f"DeepSeek checkpoint keys: missing={sorted(expected.keys() - state.keys())[:8]}, "
                             f"unexpected={sorted(state.keys() - expected.keys())[:8]}")
        backend.load_state_dict(state)
        if reader is not None:
            reader.close()
        if config.engram_layer_ids and (root / "tokenizer.json").is_file():
            from ..models.dsv4.model import build_compressed_token_map

            token_map, _ = build_compressed_token_map(root / "tokenizer.json")
            backend.model.hash = NgramHash(config, backend.model.engram_layer_ids, token_map=token_map)
    if sft_source is not None:  # a full-SFT snapshot replaces every base tensor it covers
        targets = dict(backend.state_dict())
        if sft_source.tensor_names - targets.keys():
            raise ValueError("SFT snapshot holds tensors the policy does not have")
        for name in sorted(sft_source.tensor_names):
            sft_source.copy_tensor(name, targets[name])
        for name, table in backend.model.engram_tables.items():
            for ids, values in sft_source.iter_engram_rows(f"model.engram_tables.{name}.weight"):
                table.weight.data.index_copy_(0, ids, values.to(table.weight.dtype))
    if lora_config is not None:
        inject_lora(backend, lora_config)
        adapter = _adapter(model_dir, lora_config, initial_adapter, random_init)
        if adapter is not None:
            validate_adapter_layout(backend, adapter)
            load_adapter_state(backend, adapter)
    policy = DSV41Policy(backend, trainable_scope="lora" if lora_config is not None else "all",
                         engram_offload=engram_offload)
    return policy.to_training_devices(devices, dtype)


def _is_released(root: Path) -> bool:
    index = json.loads((root / "model.safetensors.index.json").read_text(encoding="utf-8"))
    return any(name.startswith("layers.") for name in index.get("weight_map", {}))


def build_qwen_policy(model_dir, config, *, random_init: bool, devices, dtype, trainable_scope: str = "all",
                      lora_config: LoRAConfig | None = None, initial_adapter=None):
    from ..models.qwen import Qwen3MoeForCausalLM, load_qwen3_moe

    validate_qwen_config(config)
    layer_device_map(config.num_hidden_layers, devices)
    validate_available_devices(devices)
    backend = Qwen3MoeForCausalLM(config) if random_init else load_qwen3_moe(model_dir, dtype=dtype)
    if lora_config is not None:
        inject_lora(backend, lora_config)
        adapter = _adapter(model_dir, lora_config, initial_adapter, random_init)
        if adapter is not None:
            validate_adapter_layout(backend, adapter)
            load_adapter_state(backend, adapter)
    return QwenPolicy(backend, trainable_scope=trainable_scope).to_training_devices(devices, dtype)


__all__ = ["DSV41Policy", "LAST_POSITION_LOGITS_PATH", "QwenPolicy", "build_dsv41_policy", "build_qwen_policy",
           "validate_qwen_config"]
