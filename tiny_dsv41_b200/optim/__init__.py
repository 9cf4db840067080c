"""Optimizers on fused sm_100a kernels (fp32 master weights, bf16 compute copies)."""

from .adamw import FusedAdamW
from .sgd import install_sgd_in_backward

__all__ = ["FusedAdamW", "install_sgd_in_backward"]
