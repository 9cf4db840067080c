"""DeepSeek-V4.1 model family."""

from .config import DeepSeekV41Config
from .model import (CausalLMOutput, DeepSeekV41ForCausalLM, DeepSeekV41Model, DeepseekV41ForCausalLM,
                    RowShardedEmbedding, load_balancing_loss)

__all__ = ["CausalLMOutput", "DeepSeekV41Config", "DeepSeekV41ForCausalLM", "DeepSeekV41Model",
           "DeepseekV41ForCausalLM", "RowShardedEmbedding", "load_balancing_loss"]
