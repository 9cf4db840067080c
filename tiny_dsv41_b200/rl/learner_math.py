"""Numerics policy of the learner's matrix products (the ``default`` / ``bf16-no-split-k`` modes of
``dsv41_train/rl/learner_math.py:7-50``).

This library's tcgen05 GEMMs accumulate each output tile in fp32 tensor memory over the whole K
extent (no split-K, no reduced-precision reduction), so they satisfy the strict mode by
construction. The strict mode also pins the process settings that govern any PyTorch / cuBLAS
matmul a learner still issues - cuBLASLt, fp32 reductions for bf16 without split-K, fp32
matmuls at "highest" precision - and puts the previous settings back on exit.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch

STRICT = "bf16-no-split-k"


@dataclass(frozen=True)
class _MatmulSettings:
    blas: str
    reduced_precision_reduction: bool
    split_k: bool | None
    fp32_precision: str

    @classmethod
    def current(cls) -> "_MatmulSettings":
        api = torch.backends.cuda.matmul
        return cls(torch.backends.cuda.preferred_blas_library().name.lower(),
                   api.allow_bf16_reduced_precision_reduction,
                   getattr(api, "allow_bf16_reduced_precision_reduction_split_k", None),
                   torch.get_float32_matmul_precision())

    def apply(self) -> None:
        torch.backends.cuda.preferred_blas_library(self.blas)
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = (self.reduced_precision_reduction,
                                                                              self.split_k)
        torch.set_float32_matmul_precision(self.fp32_precision)

    @property
    def strict(self) -> bool:
        return (self.blas == "cublaslt" and self.reduced_precision_reduction is False and self.split_k is False
                and self.fp32_precision == "highest")

    def report(self) -> dict:
        return {"preferred_blas_library": self.blas, "bf16_reduced_precision_reduction": self.reduced_precision_reduction,
                "bf16_split_k": self.split_k, "float32_matmul_precision": self.fp32_precision,
                "native_gemm": "tcgen05, fp32 TMEM accumulation over full K, no split-K"}


def learner_math_configuration() -> dict:
    return _MatmulSettings.current().report()


def require_bf16_no_split_k() -> dict:
    settings = _MatmulSettings.current()
    if not settings.strict:
        raise ValueError("sharded response ownership requires the bf16-no-split-k learner math policy")
    return settings.report()


@contextmanager
def configure_learner_math(mode: str):
    if mode not in ("default", STRICT):
        raise ValueError("learner math mode must be default or bf16-no-split-k")
    previous = _MatmulSettings.current()
    if mode == "default":
        yield previous.report()
        return
    if previous.split_k is None:
        raise ValueError("bf16-no-split-k learner math requires PyTorch split-K control")
    try:
        _MatmulSettings("cublaslt", False, False, "highest").apply()
        yield require_bf16_no_split_k()
    finally:
        previous.apply()


__all__ = ["configure_learner_math", "learner_math_configuration", "require_bf16_no_split_k"]
