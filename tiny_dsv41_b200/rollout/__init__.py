"""Rollout-side protocols: training records, LoRA update packets and their validation."""
