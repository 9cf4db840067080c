"""Train a layer window of a released DeepSeek-V4.1 checkpoint (torchrun, one rank per GPU)."""

from tiny_dsv41_b200.train.dsv4_cli import main

if __name__ == "__main__":
    main()
