"""AdamW with fp32 master weights over bf16 compute parameters.

Each parameter (or its local FSDP/DTensor shard) gets an fp32 master copy and two moments
(fp32 by default, bf16 optionally). ``step()`` runs one fused kernel per tensor that applies
decoupled weight decay, updates the moments with bias correction (``torch.optim.AdamW``
semantics), writes the new master and the rounded bf16 parameter. With ``in_backward=True`` the
update of a parameter runs from its post-accumulate-grad hook, so gradients never accumulate for
the whole model (no global-norm clipping in that mode). ``side_stream=True`` runs those updates on
a stream of their own, so the memory-bound update of one parameter overlaps the backward GEMMs of
the next; ``finish_step()`` then orders the caller's stream after them. A gradient handed to the
side stream stays referenced until the caller's stream has waited for its update (at most
``_IN_FLIGHT`` updates behind), so its memory is never reused early and no ``record_stream`` is
needed, which keeps the step capturable in a CUDA graph. On the GPU the step count also lives in
device memory (advanced by ``begin_step``), so a captured step replays with fresh bias corrections.

On CPU the same math runs in plain PyTorch.
"""

from __future__ import annotations

import math
from collections import deque

import torch

from ..ops import ext
from ..runtime import local_tensor


_IN_FLIGHT = 4  # side-stream updates the caller's stream may run ahead of


class FusedAdamW:
    def __init__(self, params, lr: float = 1e-4, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, *, moment_dtype: torch.dtype = torch.float32,
                 in_backward: bool = False, grad_scale: float = 1.0, side_stream: bool = False,
                 side_blocks: int = 0) -> None:
        self.params = [p for p in params if p.requires_grad]
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.moment_dtype = moment_dtype
        self.grad_scale = grad_scale
        self.step_count = 0
        self.state: dict[int, dict[str, torch.Tensor]] = {}
        for p in self.params:
            local = local_tensor(p.data)
            self.state[id(p)] = {
                "master": local.detach().float().clone(),
                "m": torch.zeros(local.shape, dtype=moment_dtype, device=local.device),
                "v": torch.zeros(local.shape, dtype=moment_dtype, device=local.device),
            }
        self.in_backward = in_backward
        device = self.params[0].device if self.params else torch.device("cpu")
        self.stream = torch.cuda.Stream(device=device) if side_stream and device.type == "cuda" else None
        self._inflight: deque = deque()
        self.side_blocks = side_blocks if self.stream is not None else 0  # CTA cap beside compute (0 = none)
        self._step_t = torch.zeros(1, dtype=torch.int32, device=device) if device.type == "cuda" else None
        self._hooks = []
        self._pending_step = False
        if in_backward:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._hook))

    # -- public API ----------------------------------------------------------------------------
    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            p.grad = None

    def begin_step(self) -> None:
        """In-backward mode: advance the step counter before the backward that applies it."""
        self.step_count += 1
        if self._step_t is not None:
            self._step_t.add_(1)

    def finish_step(self) -> None:
        """Order the current stream after the updates queued on the side stream (no-op without one)."""
        if self.stream is not None:
            torch.cuda.current_stream(self.stream.device).wait_stream(self.stream)
            self._inflight.clear()

    def step(self, clip_coefficient: torch.Tensor | None = None) -> None:
        if self.in_backward:
            return
        self.begin_step()
        for p in self.params:
            if p.grad is not None:
                self._update(p, clip_coefficient)

    def state_dict(self) -> dict:
        return {"step": self.step_count, "lr": self.lr, "betas": self.betas, "eps": self.eps,
                "weight_decay": self.weight_decay,
                "state": [{k: v for k, v in self.state[id(p)].items()} for p in self.params]}

    def load_state_dict(self, state: dict) -> None:
        self.step_count = int(state["step"])
        if self._step_t is not None:
            self._step_t.fill_(self.step_count)
        for p, saved in zip(self.params, state["state"]):
            for key in ("master", "m", "v"):
                self.state[id(p)][key].copy_(saved[key])

    def remove_hooks(self) -> None:
        for hook in self._hooks:
            hook.remove()
        self._hooks = []

    # -- internals -----------------------------------------------------------------------------
    def _hook(self, p: torch.Tensor) -> None:
        if self.step_count == 0:
            self.begin_step()
        if self.stream is not None:
            main = torch.cuda.current_stream(self.stream.device)
            self.stream.wait_stream(main)
            grad = local_tensor(p.grad)
            with torch.cuda.stream(self.stream):
                self._update(p, None)
                done = torch.cuda.Event()
                done.record(self.stream)
            self._inflight.append((grad, done))
            while len(self._inflight) > _IN_FLIGHT:  # the oldest gradient may be released once the
                old, event = self._inflight.popleft()  # caller's stream is ordered after its update
                main.wait_event(event)
                del old
        else:
            self._update(p, None)
        p.grad = None

    @torch.no_grad()
    def _update(self, p: torch.Tensor, clip_coefficient: torch.Tensor | None) -> None:
        st = self.state[id(p)]
        grad = local_tensor(p.grad)
        data = local_tensor(p.data)
        beta1, beta2 = self.betas
        if data.is_cuda:
            out = data if data.dtype == torch.bfloat16 else None
            ext().adamw_step(st["master"], grad.contiguous(), st["m"], st["v"], out, self.lr, beta1, beta2,
                             self.eps, self.weight_decay, self.step_count, self.grad_scale, clip_coefficient,
                             self._step_t if self._step_t is not None and self._step_t.device == data.device else None,
                             self.side_blocks)
            if out is None:
                data.copy_(st["master"])
            return
        g = grad.float() * self.grad_scale
        if clip_coefficient is not None:
            g = g * clip_coefficient
        master = st["master"]
        master.mul_(1 - self.lr * self.weight_decay)
        m = st["m"].float().mul_(beta1).add_(g, alpha=1 - beta1)
        v = st["v"].float().mul_(beta2).addcmul_(g, g, value=1 - beta2)
        bc1 = 1 - beta1 ** self.step_count
        bc2 = 1 - beta2 ** self.step_count
        denom = (v.sqrt() / math.sqrt(bc2)).add_(self.eps)
        master.addcdiv_(m, denom, value=-self.lr / bc1)
        st["m"].copy_(m)
        st["v"].copy_(v)
        data.copy_(master)


__all__ = ["FusedAdamW"]
