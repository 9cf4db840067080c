"""Text SFT on DeepSeek-V4.1 or Qwen3-MoE checkpoints (full or LoRA).

    torchrun --nproc-per-node 8 train_sft.py --model-path MODEL --data train.jsonl \\
        --output-dir runs/sft --family qwen --mode full --ep-size 8

See ``tiny_dsv41_b200/train/sft.py`` for the flags.
"""

from tiny_dsv41_b200.train.sft import main

if __name__ == "__main__":
    main()
