"""Reinforcement learning (GRPO) stack: config, data, rewards, rollouts, algorithms, runtime."""
