"""Train the tiny DeepSeek-V4.1 model on synthetic sequences (``python train.py`` or torchrun)."""

from tiny_dsv41_b200.train.tiny import main

if __name__ == "__main__":
    main()
