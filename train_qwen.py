"""Qwen3-MoE training with context, expert and FSDP2 parallelism (torchrun, one rank per GPU)."""

from tiny_dsv41_b200.train.qwen_cli import main

if __name__ == "__main__":
    main()
