"""A rollout service backed by this library's own DeepSeek-V4.1 model, speaking the same RPC
and LoRA-packet protocol as the reference's vLLM service (``rollout.remote``).

The controller holds a frozen base model with query-LoRA adapters on ``attention.q_a`` of the
configured layers (B = 0 until the first activation). ``activate`` validates a packet, maps
``language_model.model.layers.N.attn.wq_a.lora_{A,B}.weight`` onto the adapters and returns the
packet's ``{version, digest, lineage}``. ``sample_batch`` samples every spec with a CPU generator
seeded by its ``sampling_seed`` and records the sampled-distribution log-prob of each action,
tagged with the active policy ack.

    python -m tiny_dsv41_b200.rollout.native_service --model-dir M --host 127.0.0.1 --port 29700
    (token from the DSV41_ROLLOUT_TOKEN environment variable)
"""

from __future__ import annotations

import argparse
import asyncio
import hashlib
import os
import re
from pathlib import Path

import torch

from ..rl.lora_config import DistributedLoRAConfig
from .lora_transport import policy_ack, unpack_update

_NAME = re.compile(r"language_model\.model\.layers\.(\d+)\.attn\.wq_a\.lora_([AB])\.weight\Z")


def mounted_identity(model_dir) -> dict:
    root = Path(model_dir)
    return {k: hashlib.sha256((root / n).read_bytes()).hexdigest()
            for k, n in (("config_sha256", "config.json"), ("index_sha256", "model.safetensors.index.json"))}


class NativeRolloutController:
    def __init__(self, model_dir, lora_config: DistributedLoRAConfig, *, device="cpu", dtype=torch.float32,
                 eos_token_ids=None) -> None:
        self.model_dir, self.lora_config = Path(model_dir), lora_config
        self.device, self.dtype = torch.device(device), dtype
        self.state = "created"
        self.ack = None
        self.activation_receipts: list = []
        self.base_identity = mounted_identity(model_dir)
        self.model = None
        self.eos = eos_token_ids

    async def start(self):
        from ..lora import inject_lora
        from ..models.dsv4.checkpoint import load_dsv41_backbone_prefix
        from ..models.dsv4.config import DeepSeekV41Config

        cfg = DeepSeekV41Config.from_json(self.model_dir / "config.json")
        model = load_dsv41_backbone_prefix(self.model_dir, num_layers=cfg.num_hidden_layers, device="cpu",
                                           dtype=torch.float32)
        for p in model.parameters():
            p.requires_grad_(False)
        for layer in self.lora_config.selected_layers(cfg.num_hidden_layers):
            inject_lora(model.model.layers[layer], self.lora_config.lora_config())
        model.requires_grad_(False)  # the service only samples
        if self.dtype != torch.float32:
            model.to_mixed_precision(self.dtype)
        self.model = model.to(self.device).eval()
        if self.eos is None:
            from ..rl.tokenizer import read_eos_token_ids

            self.eos = tuple(read_eos_token_ids(self.model_dir, cfg.eos_token_id))
        self.state = "paused"
        return self.state

    async def activate(self, manifest, payload):
        with torch.no_grad():
            return self._activate(manifest, payload)

    def _activate(self, manifest, payload):
        if self.state not in {"paused"}:
            raise RuntimeError("activation requires a started, paused controller")
        tensors = unpack_update(manifest, payload)
        if manifest["base_identity"] != self.base_identity:
            raise ValueError("LoRA update targets a different mounted base")
        layers = set(self.lora_config.selected_layers(len(self.model.model.layers)))
        seen = set()
        for name, value in tensors.items():
            m = _NAME.fullmatch(name)
            if m is None or int(m[1]) not in layers:
                raise ValueError(f"unsupported adapter tensor {name}")
            module = self.model.model.layers[int(m[1])].attention.q_a
            target = module.lora_a if m[2] == "A" else module.lora_b
            if tuple(target.shape) != tuple(value.shape):
                raise ValueError(f"{name} shape differs from the mounted adapter")
            target.copy_(value.to(device=target.device, dtype=target.dtype))
            seen.add(name)
        if len(seen) != 2 * len(layers):
            raise ValueError("LoRA update does not cover every configured adapter")
        self.ack = policy_ack(manifest)
        self.activation_receipts.append(dict(self.ack))
        return dict(self.ack)

    def sample_batch(self, specs):
        if self.state != "running":
            raise RuntimeError("sampling requires a resumed controller")
        return [self._sample(spec) for spec in specs]

    @torch.no_grad()
    def _sample(self, spec) -> dict:
        generator = torch.Generator(device="cpu").manual_seed(spec["sampling_seed"])
        tokens = list(spec["prompt_ids"])
        actions, logps, finish, stop = [], [], "length", 0
        for _ in range(spec["max_tokens"]):
            ids = torch.tensor([tokens + actions], dtype=torch.long, device=self.device)
            logits = self.model(ids, compute_aux_loss=False).logits[0, -1].float()
            logp = torch.log_softmax(logits / spec["temperature"], -1)
            token = int(torch.multinomial(logp.exp().cpu(), 1, generator=generator))
            actions.append(token)
            logps.append(float(logp[token]))
            if token in self.eos:
                finish, stop = "eos", 1
                break
        return {"context_token_ids": list(spec["prompt_ids"]), "action_token_ids": actions,
                "behavior_log_probs": logps, "logprob_convention": "sampled_distribution",
                "finish_reason": finish, "stop_token_count": stop,
                "generation_metrics": {"policy_ack": dict(self.ack), "request_id": spec["request_id"],
                                       "sampling_seed": spec["sampling_seed"]}}

    async def pause(self):
        self.state = "paused"
        return {"state": self.state}

    async def resume(self):
        if self.ack is None:
            raise RuntimeError("resume requires an activated adapter")
        self.state = "running"
        return {"state": self.state, "policy_ack": dict(self.ack)}

    async def close(self):
        self.state = "closed"
        return {"closed": True, "drain_complete": True}


def main(argv=None) -> None:
    from .remote import RemoteLoRAServer

    p = argparse.ArgumentParser(description="Serve native DeepSeek-V4.1 rollouts over the LoRA RPC protocol")
    p.add_argument("--model-dir", required=True)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, required=True)
    p.add_argument("--device", default="cpu")
    p.add_argument("--lora-rank", type=int, default=8)
    p.add_argument("--lora-alpha", type=float, default=8.0)
    args = p.parse_args(argv)
    controller = NativeRolloutController(args.model_dir, DistributedLoRAConfig(args.lora_rank, args.lora_alpha),
                                         device=args.device)
    with RemoteLoRAServer((args.host, args.port), os.environ["DSV41_ROLLOUT_TOKEN"], controller) as server:
        server.serve_forever()


if __name__ == "__main__":
    main()
