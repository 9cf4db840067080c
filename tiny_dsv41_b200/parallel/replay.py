"""Expert-parallel exchange replay for activation checkpointing.

With activation checkpointing a layer's forward runs twice: once in the forward pass and once
again (recompute) during backward. Re-running the MoE token exchange would move the same rows
over NVLink a second time. Instead, the first pass records what its exchanges produced (the
received expert-major rows and the combined output, plus the routing state), and the recompute
replays them: the recomputed graph gets the same tensors without any transfer, and its backward
still runs the real reverse exchanges. The causal attention forward and the small dense
projections around it (QKV and output, ``ops.linear(..., replayable=True)``) and the per-head
q / k norm + RoPE are treated the same way: their outputs (about 130 MB per layer at L 4096 for
Qwen3-30B-A3B) are kept from the first pass, so the recompute runs neither the attention kernel
nor those GEMMs nor the norm / rotation. Records are consumed in
the order they were made, so every recorded call must run in the same order in the recompute.

``checkpoint_contexts`` is passed as ``context_fn`` to ``torch.utils.checkpoint.checkpoint``
(non-reentrant): each checkpointed call gets one ``ReplayHandle``; the forward runs under its
record context, the recompute under its replay context. The handle lives as long as the
checkpoint frame, so recorded tensors are released after that layer's backward.
"""

from __future__ import annotations

import threading

_local = threading.local()


class ReplayHandle:
    def __init__(self) -> None:
        self.items: list = []
        self.cursor = 0
        # attention outputs (out, lse) of the first pass: the recompute reuses them instead of
        # running the attention forward again (its backward still gets recomputed q / k / v)
        self.attention: list = []
        self.attention_cursor = 0

    def record_attention(self, item) -> None:
        self.attention.append(item)

    def next_attention(self):
        if self.attention_cursor >= len(self.attention):
            raise RuntimeError("recompute ran more attention calls than the recorded forward")
        item = self.attention[self.attention_cursor]
        self.attention_cursor += 1
        return item

    def record(self, item) -> None:
        self.items.append(item)

    def next(self):
        if self.cursor >= len(self.items):
            raise RuntimeError("recompute issued more expert exchanges than the recorded forward")
        item = self.items[self.cursor]
        self.cursor += 1
        return item


class _Mode:
    def __init__(self, handle: ReplayHandle, mode: str) -> None:
        self.handle, self.mode = handle, mode

    def __enter__(self):
        if self.mode == "replay":
            self.handle.cursor = 0
            self.handle.attention_cursor = 0
        stack = getattr(_local, "stack", None)
        if stack is None:
            stack = _local.stack = []
        stack.append((self.handle, self.mode))
        return self

    def __exit__(self, *exc):
        _local.stack.pop()
        return False


def checkpoint_contexts():
    handle = ReplayHandle()
    return _Mode(handle, "record"), _Mode(handle, "replay")


def current():
    """(handle, "record" | "replay") of the innermost checkpointed call, or (None, None)."""
    stack = getattr(_local, "stack", None)
    return stack[-1] if stack else (None, None)


__all__ = ["ReplayHandle", "checkpoint_contexts", "current"]
