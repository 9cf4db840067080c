"""Hot ops of the framework. CUDA tensors run the sm_100a kernels of ``tiny_dsv41_b200._C``;
CPU tensors run the plain-PyTorch restatement used as the test oracle."""

from ._ext import (DeviceStatusError, StatusMonitor, available, check_status, ext, on_gpu, peer_wait_limit,
                   set_peer_wait_limit)
from .attention import causal_attention
from .fp4 import dequantize_fp4, fp4_grouped_linear
from .gemm import grouped_linear, linear, matmul_nt
from .loss import linear_cross_entropy, token_log_probs
from .moe import Routing, build_routing, combine, gather, swiglu
from .norm import rms_norm
from .quant import fake_quant, quantize_activation
from . import rope
from .rope import inv_freq, qk_norm_rope, rope_interleaved
from .router import AuxGradient, route

__all__ = [
    "AuxGradient", "DeviceStatusError", "Routing", "StatusMonitor", "available", "build_routing", "causal_attention", "check_status", "combine",
    "dequantize_fp4", "ext", "fake_quant", "fp4_grouped_linear", "gather", "grouped_linear", "inv_freq", "linear", "linear_cross_entropy", "matmul_nt", "on_gpu", "peer_wait_limit",
    "qk_norm_rope", "quantize_activation", "rms_norm", "rope_interleaved", "route", "set_peer_wait_limit", "swiglu", "token_log_probs",
]
