"""A DeepSeek-V4.1 backbone prefix with random weights, built the way the released-checkpoint
loader builds one (``checkpoint.load_dsv41_backbone_window``), without a checkpoint on disk.

Throughput runs at the Flash dimensions need the whole 40-layer model on every rank's devices
(about 290 GB of FP4 experts alone in the released layout); writing and re-reading such a
checkpoint measures the disk, not the step. Here the model is constructed on the meta device
with this rank's experts only, the routed experts are frozen as MXFP4 buffers (E2M1 codes and
E8M0 scales in the released per-32 layout) when asked, everything is then materialised in place
on the target device (the Engram tables in host memory under offload) and filled from one
seeded generator: matrices ~ N(0, std), normalisation weights 1, other vectors 0, expert codes
uniform bytes with scale 2^-6. The result is the same module tree the loader returns, so LoRA
injection, the EP dispatcher, Engram offload and mHC run unchanged.
"""

from __future__ import annotations

import torch
from torch import nn

from .config import DeepSeekV41Config
from .model import DeepSeekV41ForCausalLM, NgramHash

_FP4_SCALE = 127 - 6  # E8M0 byte of 2^-6: E2M1 values up to 6 -> weights up to about 0.09


# parameters the released checkpoint stores in fp32 and the loader keeps in fp32 ("raw" tensors)
_FP32_ISLANDS = ("attention_hc.", "moe_hc.", "attention.sinks.", "moe.router.selection_bias")


def _is_island(name: str) -> bool:
    return any(key in name for key in _FP32_ISLANDS)


def _fill(name: str, tensor: torch.Tensor, generators: dict, std: float) -> None:
    generator = generators[tensor.device.type]
    if tensor.dtype == torch.uint8:
        if name.endswith("_scale"):
            tensor.fill_(_FP4_SCALE)
        else:
            tensor.copy_(torch.randint(0, 256, tensor.shape, generator=generator, dtype=torch.uint8,
                                       device=tensor.device))
        return
    if not tensor.is_floating_point():
        tensor.zero_()
        return
    if tensor.dim() >= 2:
        # in row chunks: a Flash Engram table holds 48 M rows per rank
        step = max(1, (1 << 24) // max(1, tensor[0].numel()))
        for start in range(0, tensor.shape[0], step):
            piece = tensor[start:start + step]
            piece.copy_(torch.randn(piece.shape, generator=generator, dtype=torch.float32, device=piece.device) * std)
    elif name.endswith("norm.weight"):
        tensor.fill_(1.0)
    else:
        tensor.zero_()


@torch.no_grad()
def build_synthetic_backbone(config: DeepSeekV41Config, *, device="cpu", dtype=torch.bfloat16,
                             context_parallel=None, token_dispatcher=None, engram_mesh=None,
                             sparse_engram_gradients: bool = False, engram_offload: bool = False,
                             fp4_experts: bool = True, seed: int = 0, std: float = 0.02) -> DeepSeekV41ForCausalLM:
    """Random-weight model of ``config`` (use ``checkpoint.prefix_config`` for a layer prefix)."""
    target = torch.device(device)
    with torch.device("meta"):
        model = DeepSeekV41ForCausalLM(config, context_parallel, token_dispatcher, engram_mesh,
                                       list(range(config.num_hidden_layers)), sparse_engram_gradients,
                                       engram_offload)
        if fp4_experts:
            for layer in model.model.layers:
                routed = layer.moe.routed
                e, i, h = routed.num_experts, routed.intermediate, routed.hidden_size
                routed.freeze_fp4(torch.empty(e, i, 2, h // 2, dtype=torch.uint8),
                                  torch.empty(e, i, 2, h // 32, dtype=torch.uint8),
                                  torch.empty(e, h, i // 2, dtype=torch.uint8),
                                  torch.empty(e, h, i // 32, dtype=torch.uint8))
    # the Engram tables live in host memory under offload; everything else on the target device
    tables = model.model.engram_tables
    model.model.engram_tables = nn.ModuleDict()
    model.to_empty(device=target)
    tables.to_empty(device=torch.device("cpu") if engram_offload else target)
    model.model.engram_tables = tables
    # the checkpoint's compute dtype for everything but its fp32 islands
    for module_name, module in model.named_modules():
        for name, p in list(module.named_parameters(recurse=False)):
            full = f"{module_name}.{name}" if module_name else name
            if p.is_floating_point() and not _is_island(full) and p.dtype != dtype:
                setattr(module, name, nn.Parameter(torch.empty_like(p, dtype=dtype), requires_grad=p.requires_grad))
    generators = {"cpu": torch.Generator().manual_seed(seed)}
    if target.type == "cuda":
        generators["cuda"] = torch.Generator(device=target).manual_seed(seed)
    for module_name, module in model.named_modules():
        for name, tensor in list(module.named_parameters(recurse=False)) + list(module.named_buffers(recurse=False)):
            full = f"{module_name}.{name}" if module_name else name
            if full.startswith("model.rotary") or full.startswith("model.hash"):
                continue
            _fill(full, tensor.data, generators, std)
    rotary = model.model.rotary
    rotary.main = rotary._main_fp32.to(target)
    rotary.compressed = rotary._compressed_fp32.to(target)
    if model.model.hash is not None:
        model.model.hash = NgramHash(config, model.model.engram_layer_ids).to(target)
    if any(t.is_meta for t in list(model.parameters()) + list(model.buffers())):
        raise RuntimeError("synthetic construction left meta tensors in the model")
    return model


__all__ = ["build_synthetic_backbone"]
