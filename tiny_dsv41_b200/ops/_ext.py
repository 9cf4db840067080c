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


STATUS_CODES = {
    1: "TMA stage wait timed out", 2: "TMA stage wait timed out", 3: "accumulator wait timed out",
    4: "accumulator wait timed out", 5: "a peer rank never raised its flag (peer wait timed out)",
    6: "bad shape", 7: "index out of bounds (bounds-check build)",
}


class DeviceStatusError(RuntimeError):
    """A kernel's bounded wait gave up (or a bounds check failed); ``code`` is the status word."""

    def __init__(self, what: str, code: int) -> None:
        reason = STATUS_CODES.get(code) or ("attention / indexer pipeline wait timed out"
                                            if 300 <= code < 500 else "unknown")
        super().__init__(f"{what}: device status {code}: {reason}")
        self.code = code


def check_status(what: str = "kernel") -> None:
    """Raise if a bounded device wait gave up since the last check (synchronises the stream)."""
    code = ext().read_status()
    if code:
        raise DeviceStatusError(what, int(code))


def set_peer_wait_limit(seconds: float) -> None:
    """How long a kernel may wait for another rank's flag before it records status 5 and returns
    (process-wide; 4 s by default)."""
    ext().set_peer_wait_limit_ns(max(1, int(seconds * 1e9)))


def peer_wait_limit() -> float:
    return ext().peer_wait_limit_ns() / 1e9


class StatusMonitor:
    """Once-per-step check of the device status word in a training loop.

    ``step_end()`` enqueues, on the current stream, a copy of the word into pinned host memory and
    its reset, then waits for that copy alone: at the end of a step the stream has already drained
    (the loss was read), so the wait is one short synchronisation per step. A non-zero word raises
    :class:`DeviceStatusError` before the next step launches anything, so a rank whose peer
    stopped answering leaves the loop instead of training on a partial exchange. On a host without
    the extension or without a GPU the monitor does nothing."""

    def __init__(self, device=None) -> None:
        self.enabled = torch.cuda.is_available() and _ext is not None and (
            device is None or torch.device(device).type == "cuda")
        if not self.enabled:
            return
        with torch.cuda.device(torch.device(device) if device is not None else torch.cuda.current_device()):
            self.word = _ext.status_word()
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()

    def step_end(self, what: str = "training step") -> None:
        if not self.enabled:
            return
        self.host.copy_(self.word, non_blocking=True)
        self.word.zero_()
        self.event.record()
        self.event.synchronize()
        code = int(self.host[0])
        if code:
            raise DeviceStatusError(what, code)
