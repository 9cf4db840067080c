"""Training loops and drivers (SFT, synthetic pre-training, benchmarks)."""
