from .checkpoint import hf_tensor_names, load_qwen3_moe, save_qwen3_moe
from .config import Qwen3MoeConfig
from .model import Qwen3MoeForCausalLM, Qwen3MoeModel

__all__ = ["Qwen3MoeConfig", "Qwen3MoeForCausalLM", "Qwen3MoeModel", "hf_tensor_names", "load_qwen3_moe",
           "save_qwen3_moe"]
