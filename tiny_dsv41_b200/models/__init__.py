"""Model families: Qwen3-MoE and DeepSeek-V4.1."""
