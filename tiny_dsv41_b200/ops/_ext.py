"""Loader for the in-tree sm_100a extension ``tiny_dsv41_b200._C``.

CUDA tensors always go through the extension; if it is missing on a machine with a GPU the
call raises instead of falling back to eager PyTorch. CPU tensors use the plain PyTorch
restatement of each op (the numerical oracle used by the CPU test-suite).
"""

from __future__ import annotations

import torch

try:  # pragma: no cover - depends on the build
    from .. import _C as _ext
    _IMPORT_ERROR: Exception | None = None
except Exception as error:  # pragma: no cover
    _ext = None
    _IMPORT_ERROR = error


def available() -> bool:
    return _ext is not None


def ext():
    """Return the compiled module, raising a clear error if it was not built."""
    if _ext is None:
        raise RuntimeError(
            "tiny_dsv41_b200._C (the sm_100a kernels) is not built; run "
            "`python setup.py build_ext --inplace` (error: %r)" % (_IMPORT_ERROR,)
        )
    return _ext


def on_gpu(*tensors: torch.Tensor | None) -> bool:
    """True when the op must run its CUDA kernel (and the extension must be present)."""
    cuda = any(t is not None and t.is_cuda for t in tensors)
    if cuda:
        ext()
    return cuda


def check_status(what: str = "kernel") -> None:
    """Raise if a bounded device wait gave up since the last check (synchronises the stream)."""
    code = ext().read_status()
    if code:
        raise RuntimeError(f"{what}: device pipeline status {code} (a bounded wait timed out)")
