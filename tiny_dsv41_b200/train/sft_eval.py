"""Greedy answer evaluation through the training model's forward
(``dsv41_train/sft_eval.py:12-103``: same stopping rule, CP layout and exact-match scoring).

Every rank of an FSDP job calls with the same prompts; within a context-parallel group the
owner of the last live position contributes its vocabulary vector (all-reduce over the group),
and rank 0's argmax is broadcast so all forwards stay in lockstep.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..parallel.cp import ContextParallel


@torch.no_grad()
def greedy_generate(model, prompt_ids, *, eos_token_ids=(), max_new_tokens: int = 16, device=None) -> list[int]:
    if type(max_new_tokens) is not int or max_new_tokens < 0:
        raise ValueError("max_new_tokens must be a nonnegative integer")
    vocab = model.config.vocab_size
    tokens = list(prompt_ids)
    if not tokens or any(type(t) is not int or not 0 <= t < vocab for t in tokens):
        raise ValueError("prompt_ids must contain valid token ids")
    stops = set(eos_token_ids)
    cp = getattr(model, "context_parallel", None) or ContextParallel()
    device = device or next(model.parameters()).device
    pad = getattr(model.config, "pad_token_id", None) or 0
    dsv4 = hasattr(model.config, "hc_mult")
    options = {"compute_aux_loss": False} if dsv4 else {"output_router_logits": False}
    flags = [(m, m.training) for m in model.modules()]
    multi = dist.is_initialized() and dist.get_world_size() > 1
    generated: list[int] = []
    model.eval()
    try:
        for _ in range(max_new_tokens):
            length = len(tokens)
            padded = (length + cp.size - 1) // cp.size * cp.size
            if padded > model.config.max_position_embeddings:
                raise ValueError("generation context exceeds the model's positions")
            ids = torch.full((1, padded), pad, dtype=torch.long, device=device)
            ids[0, :length] = torch.tensor(tokens, dtype=torch.long, device=device)
            mask = torch.arange(padded, device=device).unsqueeze(0) < length
            logits = model(ids, attention_mask=mask, **options).logits
            local = padded // cp.size
            owner, position = divmod(length - 1, local)
            nxt = logits.new_zeros(vocab, dtype=torch.float32)
            if cp.rank == owner:
                nxt.copy_(logits[0, position])
            del logits
            if cp.enabled:
                dist.all_reduce(nxt, group=cp.group)
            finite = torch.isfinite(nxt).all().to(torch.int32)
            if multi:
                dist.all_reduce(finite, op=dist.ReduceOp.MIN)
            if not finite.item():
                raise RuntimeError("generation produced non-finite next-token logits")
            token_t = nxt.argmax()
            if multi:
                dist.broadcast(token_t, src=0)
            token = int(token_t.item())
            generated.append(token)
            if token in stops:
                break
            tokens.append(token)
    finally:
        for m, training in flags:
            m.training = training
    return generated


def evaluate_answers(model, examples, tokenizer, *, max_new_tokens: int = 16, device=None) -> dict:
    if not examples:
        raise ValueError("answer evaluation requires at least one example")
    records = []
    for example in examples:
        target_ids = [t for t in example["labels"] if t != -100]
        if not target_ids:
            raise ValueError("evaluation example has no supervised answer tokens")
        out = greedy_generate(model, example["prompt_ids"], eos_token_ids=tokenizer.eos_token_ids,
                              max_new_tokens=max_new_tokens, device=device)
        text = tokenizer.decode(out, skip_special_tokens=True)
        target = tokenizer.decode(target_ids, skip_special_tokens=True)
        records.append(dict(prompt_ids=list(example["prompt_ids"]), generated_ids=out, text=text,
                            target_ids=target_ids, target=target, exact_match=text == target))
    matched = sum(r["exact_match"] for r in records)
    return dict(count=len(records), exact_matches=matched, exact_match_rate=matched / len(records), examples=records)


__all__ = ["evaluate_answers", "greedy_generate"]
