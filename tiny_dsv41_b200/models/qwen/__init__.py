from .config import Qwen3MoeConfig
from .model import Qwen3MoeForCausalLM, Qwen3MoeModel

__all__ = ["Qwen3MoeConfig", "Qwen3MoeForCausalLM", "Qwen3MoeModel"]
