"""GRPO objectives and teacher-forced response scoring.

Semantics of ``dsv41_train/rl/algorithm.py:39-346``:

* ``response_log_probs`` / ``response_log_probs_batch``: log pi(action | prefix) at the sampling
  temperature for every response token (terminal EOS included), one right-padded forward for a
  batch, through the model's selected-token log-prob path when it has one.
* ``group_advantages``: (r - mean) / (population std + eps) within one prompt group.
* ``grpo_loss``: mean over responses of the per-response mean clipped surrogate
  -min(ratio * A, clip(ratio) * A), ratio = pi / behaviour, plus kl_beta * importance-weighted k3
  KL to a reference policy.
* ``decoupled_token_tis_loss``: three-policy Token-TIS surrogate with detached token weights
  min(cap, old / behaviour) on PPO(current / old).
"""

from __future__ import annotations

import math
from typing import Any, Optional, Sequence

import torch
from torch import Tensor, nn


def validate_token_ids(ids, name: str) -> list[int]:
    if isinstance(ids, Tensor):
        ids = ids.tolist()
    ids = list(ids)
    if not ids or any(type(i) is not int or i < 0 for i in ids):
        raise ValueError(f"{name} must be a nonempty list of nonnegative integers")
    return ids


def _finite(tensor: Tensor, name: str) -> None:
    if not torch.isfinite(tensor).all().item():
        raise ValueError(f"{name} contains non-finite values")


def validate_temperature(temperature: float) -> None:
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError("temperature must be finite and positive")


def input_device(model: nn.Module) -> torch.device:
    p = next(model.parameters(), None)
    if p is not None:
        return p.device
    b = next(model.buffers(), None)
    return b.device if b is not None else torch.device("cpu")


def _scores(model, tokens, token_mask, targets, temperature):
    if getattr(model, "supports_token_log_probs", False):
        scores = model(tokens, attention_mask=token_mask, target_ids=targets, target_mask=targets != -100,
                       temperature=temperature)
        scores = scores if isinstance(scores, Tensor) else scores.token_log_probs
        if scores.shape != tokens.shape:
            raise ValueError("model must return one log probability per input token")
        return scores[targets != -100].float()
    output = model(tokens, attention_mask=token_mask)
    logits = output if isinstance(output, Tensor) else output.logits
    mask = targets != -100
    chosen = targets[mask]
    if chosen.max().item() >= logits.shape[-1]:
        raise ValueError("response token ID is outside the model vocabulary")
    return (logits[mask].float() / temperature).log_softmax(-1).gather(-1, chosen[:, None]).squeeze(-1)


def response_log_probs(model: nn.Module, prompt_ids, response_ids, temperature: float = 1.0) -> Tensor:
    validate_temperature(temperature)
    prompt = validate_token_ids(prompt_ids, "prompt_ids")
    response = validate_token_ids(response_ids, "response_ids")
    hook = getattr(model, "response_log_probs", None)
    if hook is not None:
        values = hook(prompt, response, temperature)
        if not isinstance(values, Tensor) or values.shape != (len(response),):
            raise ValueError("model response_log_probs hook must return one tensor value per action")
        values = values.float()
        _finite(values, "response log probabilities")
        if bool((values > 1e-6).any()):
            raise ValueError("response log probabilities must be nonpositive")
        return values
    return response_log_probs_batch(model, [prompt], [response], temperature)[0]


def response_log_probs_batch(model: nn.Module, prompt_ids_batch, response_ids_batch, temperature: float = 1.0, *,
                             return_metadata: bool = False):
    validate_temperature(temperature)
    size = len(prompt_ids_batch)
    if not size or len(response_ids_batch) != size:
        raise ValueError("prompt and response batches require the same nonzero size")
    prompts = [validate_token_ids(p, "prompt_ids") for p in prompt_ids_batch]
    responses = [validate_token_ids(r, "response_ids") for r in response_ids_batch]
    lengths = [len(p) + len(r) - 1 for p, r in zip(prompts, responses)]
    device = input_device(model)
    tokens = torch.zeros((size, max(lengths)), dtype=torch.long, device=device)
    token_mask = torch.zeros_like(tokens, dtype=torch.bool)
    targets = torch.full_like(tokens, -100)
    for row, (p, r, n) in enumerate(zip(prompts, responses, lengths)):
        tokens[row, :n] = torch.tensor(p + r[:-1], device=device)
        token_mask[row, :n] = True
        targets[row, len(p) - 1:n] = torch.tensor(r, device=device)
    selected = _scores(model, tokens, token_mask, targets, temperature)
    _finite(selected, "response log probabilities")
    if bool((selected > 1e-6).any()):
        raise ValueError("response log probabilities must be nonpositive")
    values = list(selected.split([len(r) for r in responses]))
    if not return_metadata:
        return values
    return values, {"source": "one_padded_model_forward", "model_forward_calls": 1,
                    "batch_size": int(tokens.shape[0]), "input_shape": list(tokens.shape),
                    "input_lengths": lengths, "response_lengths": [len(r) for r in responses],
                    "valid_input_tokens": sum(lengths), "padded_input_tokens": tokens.numel() - sum(lengths),
                    "allocated_input_tokens": tokens.numel(), "response_tokens": sum(map(len, responses)),
                    "padding_side": "right"}


def group_advantages(rewards, eps: float = 1e-6) -> Tensor:
    if not math.isfinite(eps) or eps <= 0:
        raise ValueError("advantage epsilon must be finite and positive")
    values = torch.as_tensor(rewards, dtype=torch.float32).detach()
    if values.ndim != 1 or values.numel() == 0:
        raise ValueError("rewards must be a nonempty vector")
    _finite(values, "rewards")
    return (values - values.mean()) / (values.std(unbiased=False) + eps)


def grpo_loss(policy_log_probs: Sequence[Tensor], behavior_log_probs, advantages, clip_eps: float = 0.2,
              ref_log_probs: Optional[Sequence[Tensor]] = None, kl_beta: float = 0.0) -> tuple[Tensor, dict]:
    if not math.isfinite(clip_eps) or not 0 <= clip_eps < 1:
        raise ValueError("clip_eps must be finite and in [0, 1)")
    if not math.isfinite(kl_beta) or kl_beta < 0:
        raise ValueError("kl_beta must be finite and nonnegative")
    size = len(policy_log_probs)
    if size == 0 or len(behavior_log_probs) != size:
        raise ValueError("policy and behavior must contain the same nonzero number of responses")
    adv = torch.as_tensor(advantages, dtype=torch.float32).detach()
    if adv.ndim != 1 or len(adv) != size:
        raise ValueError("one scalar advantage is required per response")
    _finite(adv, "advantages")
    if ref_log_probs is not None and len(ref_log_probs) != size:
        raise ValueError("one reference log-probability vector is required per response")
    if kl_beta and ref_log_probs is None:
        raise ValueError("positive kl_beta requires reference log probabilities")
    pol, kls, clips, ratios, approx = [], [], [], [], []
    for i, current in enumerate(policy_log_probs):
        if current.ndim != 1 or current.numel() == 0:
            raise ValueError("each policy log-probability tensor must be a nonempty vector")
        current = current.float()
        _finite(current, "policy log probabilities")
        behavior = torch.as_tensor(behavior_log_probs[i], dtype=torch.float32, device=current.device).detach()
        if behavior.shape != current.shape:
            raise ValueError("behavior and policy response lengths must match")
        _finite(behavior, "behavior log probabilities")
        log_ratio = current - behavior
        ratio = torch.exp(log_ratio)
        _finite(ratio, "importance ratios (reduce policy lag or learning rate)")
        a = adv[i].to(current.device)
        pol.append(-torch.minimum(ratio * a, ratio.clamp(1 - clip_eps, 1 + clip_eps) * a).mean())
        if kl_beta:
            ref = ref_log_probs[i].to(device=current.device, dtype=torch.float32).detach()
            if ref.shape != current.shape:
                raise ValueError("reference and policy response lengths must match")
            _finite(ref, "reference log probabilities")
            delta = ref - current
            k3 = ratio * (torch.expm1(delta) - delta)
            _finite(k3, "importance-weighted reference KL")
            kls.append(k3.mean())
        else:
            kls.append(current.new_zeros(()))
        clips.append(((ratio - 1).abs() > clip_eps).float().mean().detach())
        ratios.append(ratio.mean().detach())
        approx.append((-log_ratio).mean().detach())
    policy_loss = torch.stack(pol).mean()
    kl = torch.stack(kls).mean()
    loss = policy_loss + kl_beta * kl
    _finite(loss, "GRPO loss")
    return loss, {"loss": loss.detach().item(), "policy_loss": policy_loss.detach().item(), "kl": kl.detach().item(),
                  "clip_fraction": torch.stack(clips).mean().item(), "importance_ratio": torch.stack(ratios).mean().item(),
                  "approx_kl": torch.stack(approx).mean().item()}


def decoupled_token_tis_loss(policy_log_probs, native_old_log_probs, behavior_log_probs, advantages,
                             clip_eps: float = 0.2, is_cap: float = 2.0) -> tuple[Tensor, dict]:
    if not math.isfinite(clip_eps) or not 0 <= clip_eps < 1:
        raise ValueError("clip_eps must be finite and in [0, 1)")
    if not math.isfinite(is_cap) or is_cap <= 0:
        raise ValueError("is_cap must be finite and positive")
    size = len(policy_log_probs)
    if size == 0 or len(native_old_log_probs) != size or len(behavior_log_probs) != size:
        raise ValueError("current, native-old and behavior require the same nonzero response count")
    adv = torch.as_tensor(advantages, dtype=torch.float32).detach()
    if adv.ndim != 1 or len(adv) != size:
        raise ValueError("one scalar advantage is required per response")
    _finite(adv, "advantages")
    terms, weights_all, raw_all, ratio_all, delta_all = [], [], [], [], []
    for i, current in enumerate(policy_log_probs):
        if not isinstance(current, Tensor) or current.ndim != 1 or current.numel() == 0:
            raise ValueError("each policy log-probability tensor must be a nonempty vector")
        current = current.float()
        old = torch.as_tensor(native_old_log_probs[i], dtype=torch.float32, device=current.device).detach()
        beh = torch.as_tensor(behavior_log_probs[i], dtype=torch.float32, device=current.device).detach()
        if old.shape != current.shape or beh.shape != current.shape:
            raise ValueError("native-old, behavior and policy response lengths must match")
        for name, values in (("policy", current), ("native-old", old), ("behavior", beh)):
            _finite(values, name + " log probabilities")
            if bool((values > 1e-6).any()):
                raise ValueError(name + " log probabilities must be nonpositive")
        delta = old - beh
        raw = delta.double().exp()
        _finite(raw, "raw rollout importance weights")
        if bool((raw == 0).any()):
            raise ValueError("raw rollout importance weights underflowed")
        weights = raw.clamp(max=is_cap).float().detach()
        if bool((weights == 0).any()):
            raise ValueError("training rollout importance weights underflowed")
        ratio = (current - old).exp()
        _finite(ratio, "native PPO ratios")
        if bool((ratio == 0).any()):
            raise ValueError("native PPO ratios underflowed")
        a = adv[i].to(current.device)
        surrogate = torch.minimum(ratio * a, ratio.clamp(1 - clip_eps, 1 + clip_eps) * a)
        terms.append(-(weights * surrogate).mean())
        weights_all.append(raw.clamp(max=is_cap))
        raw_all.append(raw)
        ratio_all.append(ratio.detach().double())
        delta_all.append(delta.double())
    loss = torch.stack(terms).mean()
    _finite(loss, "Token-TIS loss")
    w, raw = torch.cat(weights_all), torch.cat(raw_all)
    ratios, deltas = torch.cat(ratio_all), torch.cat(delta_all)
    total, squared, raw_total = w.sum(), w.square().sum(), raw.sum()
    ess = total.square() / squared
    dropped = (raw_total - total).clamp(min=0)
    return loss, {
        "loss": loss.detach().item(), "policy_loss": loss.detach().item(), "response_count": float(size),
        "token_count": float(w.numel()), "is_cap": float(is_cap), "is_weight_sum": total.item(),
        "is_weight_square_sum": squared.item(), "is_weight_mean": w.mean().item(), "is_weight_min": w.min().item(),
        "is_weight_max": w.max().item(), "is_raw_weight_sum": raw_total.item(), "is_raw_weight_min": raw.min().item(),
        "is_raw_weight_max": raw.max().item(), "is_clipped_tokens": float((raw > is_cap).sum().item()),
        "is_clipped_fraction": (raw > is_cap).double().mean().item(), "is_dropped_weight_mass": dropped.item(),
        "is_dropped_weight_mass_fraction": (dropped / raw_total).item(), "is_token_weight_ess": ess.item(),
        "is_token_weight_ess_fraction": ess.item() / w.numel(),
        "native_old_minus_behavior_mean": deltas.mean().item(),
        "native_old_minus_behavior_max_abs": deltas.abs().max().item(),
        "native_ppo_ratio_mean": ratios.mean().item(),
        "native_ppo_clip_fraction": ((ratios - 1).abs() > clip_eps).double().mean().item(),
    }


__all__ = ["decoupled_token_tis_loss", "group_advantages", "grpo_loss", "input_device", "response_log_probs",
           "response_log_probs_batch", "validate_temperature", "validate_token_ids"]
