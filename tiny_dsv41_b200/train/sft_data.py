"""Last-answer SFT data: chat-template encoding, supervised labels, right-padded batches.

Contract of ``dsv41_train/sft_data.py``: records are ``{"prompt", "answer"}`` or
``{"messages", "answer"}``; only the final answer through its first EOS token is supervised
(template suffixes after EOS stay masked); no truncation; batches are right-padded to a multiple
of the CP size.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..rl.tokenizer import ModelTokenizer


def encode_example(record: dict, tokenizer: ModelTokenizer, *, max_length: int, enable_thinking: bool = False) -> dict:
    if type(max_length) is not int or max_length < 2:
        raise ValueError("max_length must be an integer of at least 2")
    if not isinstance(record, dict) or set(record) not in ({"prompt", "answer"}, {"messages", "answer"}):
        raise ValueError("SFT records require exactly prompt/answer or messages/answer")
    messages = [{"role": "user", "content": record["prompt"]}] if "prompt" in record else record.get("messages")
    if not isinstance(messages, list) or not messages:
        raise ValueError("SFT messages must be a nonempty list")
    for m in messages:
        if (not isinstance(m, dict) or set(m) != {"role", "content"} or m["role"] not in ("system", "user", "assistant")
                or not isinstance(m["content"], str) or not m["content"].strip()):
            raise ValueError("SFT messages support only system/user/assistant roles with nonempty text content")
    if messages[-1]["role"] != "user":
        raise ValueError("SFT messages must end with a user message")
    prompt_ids, input_ids = tokenizer.encode_completion(
        messages, record["answer"], chat_template_kwargs={"enable_thinking": enable_thinking})
    if len(input_ids) > max_length:
        raise ValueError(f"SFT example has {len(input_ids)} tokens, exceeding max_length={max_length}; "
                         "truncation is disabled")
    start = len(prompt_ids)
    eos = next((i for i in range(start, len(input_ids)) if input_ids[i] in tokenizer.eos_token_ids), None)
    if eos is None:
        raise ValueError("completed SFT answer must contain a checkpoint EOS token")
    if eos == start:
        raise ValueError("SFT answer must contain at least one token before EOS")
    labels = [-100] * len(input_ids)
    labels[start:eos + 1] = input_ids[start:eos + 1]
    return {"input_ids": input_ids, "labels": labels, "attention_mask": [1] * len(input_ids), "prompt_ids": prompt_ids}


def load_jsonl(path, tokenizer: ModelTokenizer, *, max_length: int, enable_thinking: bool = False) -> list[dict]:
    examples = []
    with Path(path).open(encoding="utf-8") as source:
        for number, line in enumerate(source, start=1):
            if not line.strip():
                continue
            try:
                examples.append(encode_example(json.loads(line), tokenizer, max_length=max_length,
                                               enable_thinking=enable_thinking))
            except ValueError as error:
                raise ValueError(f"{path}:{number}: {error}") from error
    if not examples:
        raise ValueError(f"{path}: SFT dataset must contain at least one example")
    return examples


def collate_examples(examples: list[dict], *, pad_token_id: int, pad_to_multiple_of: int = 1) -> dict:
    if not examples:
        raise ValueError("cannot collate an empty SFT batch")
    if type(pad_token_id) is not int or pad_token_id < 0:
        raise ValueError("pad_token_id must be a nonnegative integer")
    if type(pad_to_multiple_of) is not int or pad_to_multiple_of <= 0:
        raise ValueError("pad_to_multiple_of must be a positive integer")
    length = max(len(e["input_ids"]) for e in examples)
    length = (length + pad_to_multiple_of - 1) // pad_to_multiple_of * pad_to_multiple_of
    shape = (len(examples), length)
    batch = {"input_ids": torch.full(shape, pad_token_id, dtype=torch.long),
             "labels": torch.full(shape, -100, dtype=torch.long),
             "attention_mask": torch.zeros(shape, dtype=torch.long)}
    for row, e in enumerate(examples):
        size = len(e["input_ids"])
        if not size or len(e["labels"]) != size or len(e["attention_mask"]) != size:
            raise ValueError("SFT input_ids, labels and attention_mask must have the same nonzero length")
        for name in batch:
            batch[name][row, :size] = torch.tensor(e[name], dtype=torch.long)
    return batch


__all__ = ["collate_examples", "encode_example", "load_jsonl"]
