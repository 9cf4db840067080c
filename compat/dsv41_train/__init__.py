"""Drop-in module paths of the original ``dsv41_train`` package, served by ``tiny_dsv41_b200``.

Installing this package (``pip install .``, or ``PYTHONPATH=<repo>/compat``) lets existing commands
and imports keep their names: ``python -m dsv41_train.rl.train ...`` runs this library's GRPO
runtime, and ``import dsv41_train.models.qwen`` returns this library's Qwen3-MoE module. The
command-line modules under ``dsv41_train.rl`` are real files; every other ``dsv41_train.<path>``
import is answered by an import hook that loads the module named in ``ALIASES`` and registers it
under the old name too, so both names refer to one module object.

It is a separate top-level package (not importable from the repository root by default) so that
the original package can still be imported next to this library, as the parity tests do.
"""

from __future__ import annotations

from tiny_dsv41_b200.utils.aliases import install

# original module path (below dsv41_train) -> module of this library
ALIASES = {
    "runtime": "tiny_dsv41_b200.runtime",
    "checkpoint": "tiny_dsv41_b200.checkpoint",
    "lora": "tiny_dsv41_b200.lora",
    "cp": "tiny_dsv41_b200.parallel.cp",
    "dispatch": "tiny_dsv41_b200.parallel.dispatch",
    "parallel": "tiny_dsv41_b200.parallel.meshes",
    "engram_offload": "tiny_dsv41_b200.parallel.engram_offload",
    "optim": "tiny_dsv41_b200.optim.sgd",
    "sft_data": "tiny_dsv41_b200.train.sft_data",
    "sft_eval": "tiny_dsv41_b200.train.sft_eval",
    "sft_checkpoint": "tiny_dsv41_b200.train.sft_checkpoint",
    "sft_engram": "tiny_dsv41_b200.train.sft_engram",
    "sft_export": "tiny_dsv41_b200.train.sft_export",
    "sft_source": "tiny_dsv41_b200.train.sft_source",
    "models": "tiny_dsv41_b200.models",
    "models.qwen": "tiny_dsv41_b200.models.qwen",
    "models.qwen.config": "tiny_dsv41_b200.models.qwen.config",
    "models.qwen.model": "tiny_dsv41_b200.models.qwen.model",
    "models.qwen.checkpoint": "tiny_dsv41_b200.models.qwen.checkpoint",
    "models.dsv4": "tiny_dsv41_b200.models.dsv4",
    "models.dsv4.config": "tiny_dsv41_b200.models.dsv4.config",
    "models.dsv4.model": "tiny_dsv41_b200.models.dsv4.model",
    "models.dsv4.mhc": "tiny_dsv41_b200.models.dsv4.mhc",
    "models.dsv4.checkpoint": "tiny_dsv41_b200.models.dsv4.checkpoint",
    "models.dsv4.attention": "tiny_dsv41_b200.models.dsv4.attention",
    "models.dsv4.moe": "tiny_dsv41_b200.models.dsv4.moe",
}
for _name in ("algorithm", "checkpoint", "config", "data", "engram_state", "evaluation", "family", "gsm8k",
              "learner_batch_planner", "learner_math", "lora_config", "lora_export", "manager", "parallel",
              "policy", "rewards", "rollout", "runtime", "tokenizer"):
    ALIASES[f"rl.{_name}"] = f"tiny_dsv41_b200.rl.{_name}"


install(__name__, ALIASES)
