"""GRPO objectives and teacher-forced scoring of sampled responses.

The objectives are those of ``dsv41_train/rl/algorithm.py:39-346`` (the parity test checks losses
and gradients against it); the implementation here is vectorised over a whole group: all
responses are concatenated into one token vector with a segment id per token, every token-level
quantity is computed once for the batch, and per-response means are segment sums divided by the
response lengths.

* ``response_log_probs`` / ``response_log_probs_batch``: log pi(action | prefix) at the sampling
  temperature for every response token (a terminal EOS included), one right-padded forward for
  a batch, through the model's selected-token log-prob path when it has one.
* ``group_advantages``: (r - mean) / (population std + eps) within one prompt group.
* ``grpo_loss``: mean over responses of the per-response mean clipped surrogate
  -min(ratio A, clip(ratio, 1 - eps, 1 + eps) A), ratio = pi / behaviour, plus kl_beta times the
  importance-weighted k3 estimate ratio * (exp(ref - pi) - 1 - (ref - pi)) of KL to a reference.
* ``decoupled_token_tis_loss``: three policies (current, native old, behaviour); PPO on
  current / old with detached per-token weights min(cap, old / behaviour).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
from torch import Tensor, nn

_LOGP_SLACK = 1e-6  # rounding allowance for "log-probabilities are nonpositive"


def validate_token_ids(ids, name: str) -> list[int]:
    values = ids.tolist() if isinstance(ids, Tensor) else list(ids)
    if not values or not all(type(v) is int and v >= 0 for v in values):
        raise ValueError(f"{name} must be a nonempty list of nonnegative integers")
    return values


def _require_finite(tensor: Tensor, name: str) -> None:
    if not bool(torch.isfinite(tensor).all()):
        raise ValueError(f"{name} contains non-finite values")


def _require_log_probs(tensor: Tensor, name: str) -> None:
    _require_finite(tensor, name)
    if bool((tensor > _LOGP_SLACK).any()):
        raise ValueError(f"{name} must be nonpositive")


def validate_temperature(temperature: float) -> None:
    if not (math.isfinite(temperature) and temperature > 0):
        raise ValueError("temperature must be finite and positive")


def input_device(model: nn.Module) -> torch.device:
    for tensor in (*model.parameters(), *model.buffers()):
        return tensor.device
    return torch.device("cpu")


# -- scoring --------------------------------------------------------------------------------------
def _selected_log_probs(model, tokens, token_mask, targets, temperature) -> Tensor:
    """Log-probabilities of the target tokens (positions where targets != -100), in order."""
    picked = targets != -100
    if getattr(model, "supports_token_log_probs", False):
        out = model(tokens, attention_mask=token_mask, target_ids=targets, target_mask=picked,
                    temperature=temperature)
        per_token = out if isinstance(out, Tensor) else out.token_log_probs
        if per_token.shape != tokens.shape:
            raise ValueError("model must return one log probability per input token")
        return per_token[picked].float()
    out = model(tokens, attention_mask=token_mask)
    logits = (out if isinstance(out, Tensor) else out.logits)[picked].float()
    wanted = targets[picked]
    if int(wanted.max()) >= logits.shape[-1]:
        raise ValueError("response token ID is outside the model vocabulary")
    return torch.log_softmax(logits / temperature, dim=-1).gather(-1, wanted.unsqueeze(-1)).squeeze(-1)


def response_log_probs(model: nn.Module, prompt_ids, response_ids, temperature: float = 1.0) -> Tensor:
    validate_temperature(temperature)
    prompt = validate_token_ids(prompt_ids, "prompt_ids")
    response = validate_token_ids(response_ids, "response_ids")
    hook = getattr(model, "response_log_probs", None)
    if hook is None:
        return response_log_probs_batch(model, [prompt], [response], temperature)[0]
    values = hook(prompt, response, temperature)
    if not isinstance(values, Tensor) or tuple(values.shape) != (len(response),):
        raise ValueError("model response_log_probs hook must return one tensor value per action")
    values = values.float()
    _require_log_probs(values, "response log probabilities")
    return values


def response_log_probs_batch(model: nn.Module, prompt_ids_batch, response_ids_batch, temperature: float = 1.0, *,
                             return_metadata: bool = False):
    """One right-padded teacher-forced forward: row i holds prompt_i + response_i[:-1] and targets
    response_i from the last prompt position on."""
    validate_temperature(temperature)
    if not prompt_ids_batch or len(prompt_ids_batch) != len(response_ids_batch):
        raise ValueError("prompt and response batches require the same nonzero size")
    prompts = [validate_token_ids(p, "prompt_ids") for p in prompt_ids_batch]
    responses = [validate_token_ids(r, "response_ids") for r in response_ids_batch]
    rows = [p + r[:-1] for p, r in zip(prompts, responses)]
    lengths = [len(row) for row in rows]
    width = max(lengths)
    device = input_device(model)
    tokens = torch.tensor([row + [0] * (width - len(row)) for row in rows], dtype=torch.long, device=device)
    positions = torch.arange(width, device=device)
    token_mask = positions.unsqueeze(0) < torch.tensor(lengths, device=device).unsqueeze(1)
    target_rows = [[-100] * (len(p) - 1) + r + [-100] * (width - len(p) - len(r) + 1)
                   for p, r in zip(prompts, responses)]
    targets = torch.tensor(target_rows, dtype=torch.long, device=device)
    selected = _selected_log_probs(model, tokens, token_mask, targets, temperature)
    _require_log_probs(selected, "response log probabilities")
    per_response = list(selected.split([len(r) for r in responses]))
    if not return_metadata:
        return per_response
    used, response_tokens = sum(lengths), sum(len(r) for r in responses)
    return per_response, {
        "source": "one_padded_model_forward", "model_forward_calls": 1, "batch_size": len(rows),
        "input_shape": [len(rows), width], "input_lengths": lengths, "response_lengths": [len(r) for r in responses],
        "valid_input_tokens": used, "padded_input_tokens": len(rows) * width - used,
        "allocated_input_tokens": len(rows) * width, "response_tokens": response_tokens, "padding_side": "right",
    }


def group_advantages(rewards, eps: float = 1e-6) -> Tensor:
    if not (math.isfinite(eps) and eps > 0):
        raise ValueError("advantage epsilon must be finite and positive")
    r = torch.as_tensor(rewards, dtype=torch.float32).detach()
    if r.ndim != 1 or r.numel() == 0:
        raise ValueError("rewards must be a nonempty vector")
    _require_finite(r, "rewards")
    return (r - r.mean()) / (r.std(unbiased=False) + eps)


# -- flattened groups -----------------------------------------------------------------------------
class _Flat:
    """The responses of one loss call as one token vector: ``segment[t]`` is the response of token
    t, ``lengths`` the tokens per response."""

    def __init__(self, current: Sequence[Tensor]) -> None:
        if not len(current):
            raise ValueError("policy and behavior must contain the same nonzero number of responses")
        for values in current:
            if not isinstance(values, Tensor) or values.ndim != 1 or values.numel() == 0:
                raise ValueError("each policy log-probability tensor must be a nonempty vector")
        self.count = len(current)
        self.device = current[0].device
        self.shapes = [values.shape for values in current]
        self.lengths = torch.tensor([values.numel() for values in current], device=self.device)
        self.segment = torch.repeat_interleave(torch.arange(self.count, device=self.device), self.lengths)
        self.values = torch.cat([values.float() for values in current])

    def aligned(self, others, message: str, dtype=torch.float32) -> Tensor:
        parts = [torch.as_tensor(o, dtype=dtype, device=self.device).detach() for o in others]
        if len(parts) != self.count or any(p.shape != s for p, s in zip(parts, self.shapes)):
            raise ValueError(message)
        return torch.cat(parts)

    def per_token(self, per_response: Tensor) -> Tensor:
        return per_response.to(self.device)[self.segment]

    def mean_of_means(self, token_values: Tensor) -> Tensor:
        """Mean over responses of each response's token mean."""
        sums = torch.zeros(self.count, dtype=token_values.dtype, device=self.device)
        sums = sums.index_add(0, self.segment, token_values)
        return (sums / self.lengths.to(token_values.dtype)).mean()


def _advantages(advantages, count: int) -> Tensor:
    adv = torch.as_tensor(advantages, dtype=torch.float32).detach()
    if adv.ndim != 1 or adv.numel() != count:
        raise ValueError("one scalar advantage is required per response")
    _require_finite(adv, "advantages")
    return adv


def _clipped_surrogate(ratio: Tensor, adv: Tensor, clip_eps: float) -> Tensor:
    return torch.minimum(ratio * adv, ratio.clamp(1 - clip_eps, 1 + clip_eps) * adv)


def _check_clip(clip_eps: float) -> None:
    if not (math.isfinite(clip_eps) and 0 <= clip_eps < 1):
        raise ValueError("clip_eps must be finite and in [0, 1)")


def grpo_loss(policy_log_probs: Sequence[Tensor], behavior_log_probs, advantages, clip_eps: float = 0.2,
              ref_log_probs: Optional[Sequence[Tensor]] = None, kl_beta: float = 0.0) -> tuple[Tensor, dict]:
    _check_clip(clip_eps)
    if not (math.isfinite(kl_beta) and kl_beta >= 0):
        raise ValueError("kl_beta must be finite and nonnegative")
    if len(policy_log_probs) == 0 or len(behavior_log_probs) != len(policy_log_probs):
        raise ValueError("policy and behavior must contain the same nonzero number of responses")
    flat = _Flat(policy_log_probs)
    adv = _advantages(advantages, flat.count)
    if ref_log_probs is not None and len(ref_log_probs) != flat.count:
        raise ValueError("one reference log-probability vector is required per response")
    if kl_beta and ref_log_probs is None:
        raise ValueError("positive kl_beta requires reference log probabilities")
    current = flat.values
    _require_finite(current, "policy log probabilities")
    behavior = flat.aligned(behavior_log_probs, "behavior and policy response lengths must match")
    _require_finite(behavior, "behavior log probabilities")
    log_ratio = current - behavior
    ratio = log_ratio.exp()
    _require_finite(ratio, "importance ratios (reduce policy lag or learning rate)")
    policy_loss = -flat.mean_of_means(_clipped_surrogate(ratio, flat.per_token(adv), clip_eps))
    if kl_beta:
        ref = flat.aligned(ref_log_probs, "reference and policy response lengths must match")
        _require_finite(ref, "reference log probabilities")
        gap = ref - current
        k3 = ratio * (torch.expm1(gap) - gap)
        _require_finite(k3, "importance-weighted reference KL")
        kl = flat.mean_of_means(k3)
    else:
        kl = current.new_zeros(())
    loss = policy_loss + kl_beta * kl
    _require_finite(loss, "GRPO loss")
    with torch.no_grad():
        stats = {
            "loss": loss.item(), "policy_loss": policy_loss.item(), "kl": kl.item(),
            "clip_fraction": flat.mean_of_means(((ratio - 1).abs() > clip_eps).float()).item(),
            "importance_ratio": flat.mean_of_means(ratio).item(),
            "approx_kl": flat.mean_of_means(-log_ratio).item(),
        }
    return loss, stats


def decoupled_token_tis_loss(policy_log_probs, native_old_log_probs, behavior_log_probs, advantages,
                             clip_eps: float = 0.2, is_cap: float = 2.0) -> tuple[Tensor, dict]:
    _check_clip(clip_eps)
    if not (math.isfinite(is_cap) and is_cap > 0):
        raise ValueError("is_cap must be finite and positive")
    count = len(policy_log_probs)
    if count == 0 or len(native_old_log_probs) != count or len(behavior_log_probs) != count:
        raise ValueError("current, native-old and behavior require the same nonzero response count")
    flat = _Flat(policy_log_probs)
    adv = _advantages(advantages, count)
    message = "native-old, behavior and policy response lengths must match"
    current = flat.values
    old = flat.aligned(native_old_log_probs, message)
    behavior = flat.aligned(behavior_log_probs, message)
    for name, values in (("policy", current), ("native-old", old), ("behavior", behavior)):
        _require_log_probs(values, name + " log probabilities")
    gap = old - behavior
    raw = gap.double().exp()  # rollout importance weights old / behaviour, before the cap
    _require_finite(raw, "raw rollout importance weights")
    if bool((raw == 0).any()):
        raise ValueError("raw rollout importance weights underflowed")
    capped = raw.clamp(max=is_cap)
    weights = capped.float().detach()
    if bool((weights == 0).any()):
        raise ValueError("training rollout importance weights underflowed")
    ratio = (current - old).exp()
    _require_finite(ratio, "native PPO ratios")
    if bool((ratio == 0).any()):
        raise ValueError("native PPO ratios underflowed")
    loss = -flat.mean_of_means(weights * _clipped_surrogate(ratio, flat.per_token(adv), clip_eps))
    _require_finite(loss, "Token-TIS loss")
    with torch.no_grad():
        ratios, gaps = ratio.double(), gap.double()
        total, squared, raw_total = capped.sum(), capped.square().sum(), raw.sum()
        ess = total.square() / squared
        dropped = (raw_total - total).clamp(min=0)
        tokens = capped.numel()
        stats = {
            "loss": loss.item(), "policy_loss": loss.item(), "response_count": float(count),
            "token_count": float(tokens), "is_cap": float(is_cap), "is_weight_sum": total.item(),
            "is_weight_square_sum": squared.item(), "is_weight_mean": capped.mean().item(),
            "is_weight_min": capped.min().item(), "is_weight_max": capped.max().item(),
            "is_raw_weight_sum": raw_total.item(), "is_raw_weight_min": raw.min().item(),
            "is_raw_weight_max": raw.max().item(), "is_clipped_tokens": float((raw > is_cap).sum().item()),
            "is_clipped_fraction": (raw > is_cap).double().mean().item(), "is_dropped_weight_mass": dropped.item(),
            "is_dropped_weight_mass_fraction": (dropped / raw_total).item(), "is_token_weight_ess": ess.item(),
            "is_token_weight_ess_fraction": ess.item() / tokens,
            "native_old_minus_behavior_mean": gaps.mean().item(),
            "native_old_minus_behavior_max_abs": gaps.abs().max().item(),
            "native_ppo_ratio_mean": ratios.mean().item(),
            "native_ppo_clip_fraction": ((ratios - 1).abs() > clip_eps).double().mean().item(),
        }
    return loss, stats


__all__ = ["decoupled_token_tis_loss", "group_advantages", "grpo_loss", "input_device", "response_log_probs",
           "response_log_probs_batch", "validate_temperature", "validate_token_ids"]
