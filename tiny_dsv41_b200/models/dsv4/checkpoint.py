"""Released DeepSeek-V4.1 checkpoint loading (FP8 dense weights, FP4 experts, FP8 Engram rows).

Tensor-name map, quantisation layouts, prefix/window configs and the ``layer_loaded`` callback
follow ``dsv41_train/models/dsv4/checkpoint.py:319-560``: the model is built on the meta device,
each layer is read (only this rank's expert range and Engram rows), dequantised and assigned,
then handed to ``layer_loaded`` (LoRA injection / FSDP wrapping per layer).
``write_released_checkpoint`` produces the same layout from a native model (tests and
synthetic benchmarks).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Callable

import torch

from ...utils.quant import (dequantize_fp4_rows, dequantize_fp8_blocks, dequantize_fp8_rows, quantize_fp4_rows,
                            quantize_fp8_blocks, quantize_fp8_rows)
from ...utils.safetensors_io import ShardedSafeTensorReader, save_sharded
from .config import DeepSeekV41Config
from .model import DeepSeekV41ForCausalLM, NgramHash, build_compressed_token_map


def _prefix_config(folder: Path, num_layers: int) -> DeepSeekV41Config:
    return prefix_config(DeepSeekV41Config.from_json(folder / "config.json"), num_layers)


def prefix_config(full: DeepSeekV41Config, num_layers: int) -> DeepSeekV41Config:
    """The configuration of the first ``num_layers`` real layers of a full backbone."""
    if not 1 <= num_layers <= full.num_hidden_layers:
        raise NotImplementedError(f"a full checkpoint prefix supports one to {full.num_hidden_layers} real layers")
    values = full.to_dict()
    values["num_hidden_layers"] = num_layers
    values["compress_ratios"] = full.compress_ratios[:num_layers]
    values["kv_source_layer_ids"] = [x for x in full.kv_source_layer_ids if x < num_layers]
    values["index_source_layer_ids"] = [x for x in full.index_source_layer_ids if x < num_layers]
    src = full.candidate_source_layer_id
    values["candidate_source_layer_id"] = src if 0 <= src < num_layers else -1
    engram = [(i, rows) for i, rows in zip(full.engram_layer_ids, full.engram_num_embeddings) if i < num_layers]
    values["engram_layer_ids"] = [i for i, _ in engram]
    values["engram_num_embeddings"] = [rows for _, rows in engram]
    return DeepSeekV41Config(**values)


# (native name suffix, released tensor stem, kind) for per-layer dense tensors;
# kind: "raw" read as is (fp32 islands), "cast" read and cast, "fp8" 32x32 block-scaled FP8
_LAYER_MAP = (
    ("attention_hc.base", "hc_attn_base", "raw"), ("attention_hc.fn", "hc_attn_fn", "raw"),
    ("attention_hc.scale", "hc_attn_scale", "raw"), ("moe_hc.base", "hc_ffn_base", "raw"),
    ("moe_hc.fn", "hc_ffn_fn", "raw"), ("moe_hc.scale", "hc_ffn_scale", "raw"),
    ("attention.sinks.weight", "attn.attn_sink", "raw"),
    ("attention.q_a.weight", "attn.wq_a", "fp8"), ("attention.q_norm.weight", "attn.q_norm.weight", "cast"),
    ("attention.q_b.weight", "attn.wq_b", "fp8"), ("attention.kv_proj.weight", "attn.wkv", "fp8"),
    ("attention.kv_norm.weight", "attn.kv_norm.weight", "cast"), ("attention.o_a.weight", "attn.wo_a", "fp8"),
    ("attention.o_b.weight", "attn.wo_b", "fp8"), ("input_norm.weight", "attn_norm.weight", "cast"),
    ("post_attention_norm.weight", "ffn_norm.weight", "cast"), ("moe.router.weight", "ffn.gate.weight", "cast"),
    ("moe.router.selection_bias", "ffn.gate.bias", "raw"),
    ("moe.shared.gate.weight", "ffn.shared_experts.w1", "fp8"), ("moe.shared.up.weight", "ffn.shared_experts.w3", "fp8"),
    ("moe.shared.down.weight", "ffn.shared_experts.w2", "fp8"),
)


def _assign(module: torch.nn.Module, state: dict) -> None:
    result = module.load_state_dict(state, strict=True, assign=True)
    if result.missing_keys or result.unexpected_keys:
        raise RuntimeError(f"checkpoint mismatch: missing={result.missing_keys[:5]}, unexpected={result.unexpected_keys[:5]}")


def _load_engram_rows(ckpt, source, table, *, device, dtype):
    rows, width = table.global_num_embeddings, table.embedding_dim
    if width % 32:
        raise ValueError("released Engram row width must be divisible by 32")
    for suffix, shape, storage in (("weight", [rows, width], "F8_E4M3"), ("scale", [rows, width // 32], "F8_E8M0")):
        meta = ckpt.metadata(f"{source}.engram.embed.{suffix}")
        if meta["shape"] != shape or meta["dtype"] != storage:
            raise ValueError(f"invalid released Engram layout for {source}.engram.embed.{suffix}")
    weight = torch.empty(table.weight.shape, device=device, dtype=dtype)
    for start in range(table.row_start, table.row_stop, 131072):
        stop = min(start + 131072, table.row_stop)
        values = ckpt.tensor_rows(f"{source}.engram.embed.weight", start, stop, device)
        scales = ckpt.tensor_rows(f"{source}.engram.embed.scale", start, stop, device)
        weight[start - table.row_start:stop - table.row_start].copy_(dequantize_fp8_rows(values, scales, dtype=dtype))
    return weight


def load_dsv41_backbone_window(folder, *, start_layer: int = 0, num_layers: int = 1, device="cpu",
                               dtype=torch.bfloat16, context_parallel=None, token_dispatcher=None, engram_mesh=None,
                               sparse_engram_gradients: bool = False,
                               layer_loaded: Callable | None = None, engram_weights=None,
                               engram_offload: bool = False, fp4_experts: bool = False,
                               cache_quantization: str | None = None) -> DeepSeekV41ForCausalLM:
    """``fp4_experts`` keeps the routed experts as frozen MXFP4 codes + E8M0 scales (uint8 buffers
    that the grouped GEMMs read packed) instead of dequantising them to ``dtype`` at load. ``cache_quantization``
    ("none" / "hf") overrides the checkpoint config's setting."""
    folder = Path(folder)
    if engram_offload and engram_weights is not None:
        raise ValueError("trainable CPU offload cannot reuse frozen shared Engram weights")
    if start_layer == 0:
        config = _prefix_config(folder, num_layers)
        layer_ids = list(range(num_layers))
    else:
        config = DeepSeekV41Config.from_json(folder / "config.json")
        stop = start_layer + num_layers
        if num_layers < 1 or not 0 < start_layer < stop <= config.num_hidden_layers:
            raise ValueError("the layer window must be inside the checkpoint backbone")
        if start_layer not in config.kv_source_layer_ids:
            raise ValueError("a non-prefix layer window must start at a KV source layer")
        layer_ids = list(range(start_layer, stop))
    if cache_quantization is not None:
        config = DeepSeekV41Config.from_dict({**config.to_dict(), "cache_quantization": cache_quantization})
    with torch.device("meta"):
        model = DeepSeekV41ForCausalLM(config, context_parallel, token_dispatcher, engram_mesh, layer_ids,
                                       sparse_engram_gradients, engram_offload)
    target = torch.device(device)
    rotary = model.model.rotary
    rotary.main = rotary._main_fp32.to(target)
    rotary.compressed = rotary._compressed_fp32.to(target)
    with ShardedSafeTensorReader(folder) as ckpt:
        read = lambda name: ckpt.tensor(name, target)  # noqa: E731

        def fp8(stem):
            return dequantize_fp8_blocks(read(f"{stem}.weight"), read(f"{stem}.scale"), dtype=dtype)

        _assign(model.model.embedding, {"weight": read("embed.weight").to(dtype)})
        _assign(model.model.norm, {"weight": read("norm.weight").to(dtype)})
        _assign(model.lm_head, {"weight": read("head.weight").to(dtype)})
        for layer in model.model.layers:
            lid = layer.layer_id
            src = f"layers.{lid}"
            state = {}
            for name, stem, kind in _LAYER_MAP:
                if kind == "fp8":
                    value = fp8(f"{src}.{stem}")
                else:
                    value = read(f"{src}.{stem}")
                    if kind == "cast":
                        value = value.to(dtype)
                state[name] = value
            state["attention.o_a.weight"] = state["attention.o_a.weight"].view(config.o_groups, config.o_lora_rank, -1)
            routed = layer.moe.routed
            experts = range(routed.expert_start, routed.expert_start + routed.num_experts)
            if fp4_experts:
                e, i, h = routed.num_experts, routed.intermediate, routed.hidden_size
                raw = lambda name: read(name).view(torch.uint8)  # noqa: E731
                codes = {"gate_up_fp4": torch.empty(e, i, 2, h // 2, dtype=torch.uint8, device=target),
                         "gate_up_scale": torch.empty(e, i, 2, h // 32, dtype=torch.uint8, device=target),
                         "down_fp4": torch.empty(e, h, i // 2, dtype=torch.uint8, device=target),
                         "down_scale": torch.empty(e, h, i // 32, dtype=torch.uint8, device=target)}
                for local, gid in enumerate(experts):
                    prefix = f"{src}.ffn.experts.{gid}"
                    codes["gate_up_fp4"][local, :, 0].copy_(raw(f"{prefix}.w1.weight"))
                    codes["gate_up_fp4"][local, :, 1].copy_(raw(f"{prefix}.w3.weight"))
                    codes["gate_up_scale"][local, :, 0].copy_(raw(f"{prefix}.w1.scale"))
                    codes["gate_up_scale"][local, :, 1].copy_(raw(f"{prefix}.w3.scale"))
                    codes["down_fp4"][local].copy_(raw(f"{prefix}.w2.weight"))
                    codes["down_scale"][local].copy_(raw(f"{prefix}.w2.scale"))
                routed.freeze_fp4(*codes.values())
                state.update({f"moe.routed.{k}": v for k, v in codes.items()})
            else:
                gate_up = torch.empty(routed.gate_up.shape, device=target, dtype=dtype)
                down = torch.empty(routed.down.shape, device=target, dtype=dtype)
                for local, gid in enumerate(experts):
                    prefix = f"{src}.ffn.experts.{gid}"
                    w = lambda n: dequantize_fp4_rows(read(f"{prefix}.{n}.weight"), read(f"{prefix}.{n}.scale"), dtype=dtype)  # noqa: E731
                    gate_up[local, :, 0].copy_(w("w1"))
                    gate_up[local, :, 1].copy_(w("w3"))
                    down[local].copy_(w("w2"))
                state["moe.routed.gate_up"] = gate_up
                state["moe.routed.down"] = down
            comp = layer.attention.compressor
            if comp is not None:
                state["attention.compressor.kv_proj.weight"] = read(f"{src}.attn.compressor.wkv.weight").to(dtype)
                if comp.gate_proj is not None:
                    state["attention.compressor.gate_proj.weight"] = read(f"{src}.attn.compressor.wgate.weight").to(dtype)
                state["attention.compressor.norm.weight"] = read(f"{src}.attn.compressor.norm.weight").to(dtype)
            idx = layer.attention.indexer
            if idx is not None:
                state["attention.indexer.q_proj.weight"] = fp8(f"{src}.attn.indexer.wq_b")
                state["attention.indexer.weight_proj.weight"] = read(f"{src}.attn.indexer.weights_proj.weight").to(dtype)
                if idx.owns_keys:
                    state["attention.indexer.k_proj.weight"] = read(f"{src}.attn.indexer.wk.weight").to(dtype)
                    state["attention.indexer.k_norm.weight"] = read(f"{src}.attn.indexer.k_norm.weight").to(dtype)
            if layer.engram is not None:
                table = model.model.engram_tables[str(lid)]
                if engram_weights is not None:
                    table_weight = engram_weights[str(lid)]
                else:
                    table_weight = _load_engram_rows(ckpt, src, table, dtype=dtype,
                                                     device=torch.device("cpu") if engram_offload else target)
                _assign(table, {"weight": table_weight})
                state["engram.q_weight"] = read(f"{src}.engram.q_weight").to(dtype)
                state["engram.k_weight"] = read(f"{src}.engram.k_weight").to(dtype)
                state["engram.proj.weight"] = fp8(f"{src}.engram.wkv")
            _assign(layer, state)
            if layer_loaded is not None:
                layer_loaded(layer)
    if model.model.hash is not None:
        tokenizer = folder / "tokenizer.json"
        if tokenizer.exists():
            token_map, compressed = build_compressed_token_map(tokenizer)
            if compressed != config.engram_compressed_vocab_size:
                raise ValueError(f"tokenizer-derived compressed vocabulary size ({compressed}) does not match "
                                 f"the model config ({config.engram_compressed_vocab_size})")
        else:
            token_map = None
        model.model.hash = NgramHash(config, model.model.engram_layer_ids, token_map=token_map).to(target)
    if any(p.is_meta for p in model.parameters()):
        raise RuntimeError("checkpoint loading left meta parameters in the model")
    return model


def load_dsv41_backbone_prefix(folder, *, num_layers: int = 1, **kwargs) -> DeepSeekV41ForCausalLM:
    return load_dsv41_backbone_window(folder, start_layer=0, num_layers=num_layers, **kwargs)


@torch.no_grad()
def write_released_checkpoint(model: DeepSeekV41ForCausalLM, folder, *, shard_size: int = 2 ** 30) -> None:
    """Write a (full, unsharded) native model in the released tensor layout and quantisation."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    cfg = model.config
    out: dict[str, torch.Tensor] = {}

    def put_fp8(stem, w):
        q, s = quantize_fp8_blocks(w.detach().float().cpu())
        out[f"{stem}.weight"], out[f"{stem}.scale"] = q, s

    out["embed.weight"] = model.model.embedding.weight.detach().cpu().to(torch.bfloat16)
    out["norm.weight"] = model.model.norm.weight.detach().cpu().to(torch.bfloat16)
    out["head.weight"] = model.lm_head.weight.detach().cpu().to(torch.bfloat16)
    for layer in model.model.layers:
        src = f"layers.{layer.layer_id}"
        state = layer.state_dict()
        state["attention.o_a.weight"] = state["attention.o_a.weight"].reshape(cfg.o_groups * cfg.o_lora_rank, -1)
        for name, stem, kind in _LAYER_MAP:
            value = state[name]
            if kind == "fp8":
                put_fp8(f"{src}.{stem}", value)
            else:
                out[f"{src}.{stem}"] = value.detach().cpu().float() if kind == "raw" else value.detach().cpu().to(torch.bfloat16)
        routed = layer.moe.routed
        for local in range(routed.num_experts):
            gid = routed.expert_start + local
            for proj, w in (("w1", routed.gate_up[local, :, 0]), ("w3", routed.gate_up[local, :, 1]),
                            ("w2", routed.down[local])):
                q, s = quantize_fp4_rows(w.detach().float().cpu())
                out[f"{src}.ffn.experts.{gid}.{proj}.weight"], out[f"{src}.ffn.experts.{gid}.{proj}.scale"] = q, s
        comp = layer.attention.compressor
        if comp is not None:
            out[f"{src}.attn.compressor.wkv.weight"] = comp.kv_proj.weight.detach().cpu().to(torch.bfloat16)
            if comp.gate_proj is not None:
                out[f"{src}.attn.compressor.wgate.weight"] = comp.gate_proj.weight.detach().cpu().to(torch.bfloat16)
            out[f"{src}.attn.compressor.norm.weight"] = comp.norm.weight.detach().cpu().to(torch.bfloat16)
        idx = layer.attention.indexer
        if idx is not None:
            put_fp8(f"{src}.attn.indexer.wq_b", idx.q_proj.weight)
            out[f"{src}.attn.indexer.weights_proj.weight"] = idx.weight_proj.weight.detach().cpu().to(torch.bfloat16)
            if idx.owns_keys:
                out[f"{src}.attn.indexer.wk.weight"] = idx.k_proj.weight.detach().cpu().to(torch.bfloat16)
                out[f"{src}.attn.indexer.k_norm.weight"] = idx.k_norm.weight.detach().cpu().to(torch.bfloat16)
        if layer.engram is not None:
            table = model.model.engram_tables[str(layer.layer_id)]
            q, s = quantize_fp8_rows(table.weight.detach().float().cpu())
            out[f"{src}.engram.embed.weight"], out[f"{src}.engram.embed.scale"] = q, s
            out[f"{src}.engram.q_weight"] = layer.engram.q_weight.detach().cpu().to(torch.bfloat16)
            out[f"{src}.engram.k_weight"] = layer.engram.k_weight.detach().cpu().to(torch.bfloat16)
            put_fp8(f"{src}.engram.wkv", layer.engram.proj.weight)
    save_sharded(out, folder, shard_size)
    (folder / "config.json").write_text(json.dumps(cfg.to_dict(), indent=1))


__all__ = ["load_dsv41_backbone_prefix", "load_dsv41_backbone_window", "write_released_checkpoint"]
