"""Drop-in module paths of the original ``rollout_manager`` package, served by
``tiny_dsv41_b200.rollout`` (the protocols, records, coordinator and CLI that an external rollout
service shares with the learner). ``python -m rollout_manager`` runs this library's rollout CLI."""

from tiny_dsv41_b200.utils.aliases import install

ALIASES = {name: f"tiny_dsv41_b200.rollout.{name}" for name in (
    "contracts", "coordinator", "training", "events", "telemetry", "benchmark_training", "generation_training",
    "cli")}
ALIASES.update({
    "backends": "tiny_dsv41_b200.rollout",
    "backends.pytorch_rl": "tiny_dsv41_b200.rollout.backends",
    "backends.vllm_lora_remote": "tiny_dsv41_b200.rollout.remote",
    "backends.vllm_lora_transport": "tiny_dsv41_b200.rollout.lora_transport",
    "backends.qwen_kv_cache": "tiny_dsv41_b200.models.qwen.generation",
    "analysis": "tiny_dsv41_b200.utils",
    "analysis.stage_timings": "tiny_dsv41_b200.utils.stage_timings",
})
install(__name__, ALIASES)
