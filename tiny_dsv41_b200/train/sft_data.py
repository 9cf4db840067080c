"""Last-answer SFT data: chat-template encoding, supervised labels and right-padded batches.

The record contract is the one of ``dsv41_train/sft_data.py`` (datasets are shared): each JSONL
record is ``{"prompt", "answer"}`` or ``{"messages", "answer"}``. Only the final answer is
supervised, from its first token through its first EOS token (anything the template appends
after the EOS stays masked); nothing is truncated; batches are right-padded to a multiple of the
context-parallel degree.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..rl.tokenizer import ModelTokenizer

IGNORE = -100
_ROLES = ("system", "user", "assistant")
_RECORD_SHAPES = ({"prompt", "answer"}, {"messages", "answer"})


def _conversation(record) -> list[dict]:
    if not isinstance(record, dict) or set(record) not in _RECORD_SHAPES:
        raise ValueError("SFT records require exactly prompt/answer or messages/answer")
    turns = [{"role": "user", "content": record["prompt"]}] if "prompt" in record else record["messages"]
    if not isinstance(turns, list) or not turns:
        raise ValueError("SFT messages must be a nonempty list")
    for turn in turns:
        valid = (isinstance(turn, dict) and set(turn) == {"role", "content"} and turn["role"] in _ROLES
                 and isinstance(turn["content"], str) and turn["content"].strip() != "")
        if not valid:
            raise ValueError("SFT messages support only system/user/assistant roles with nonempty text content")
    if turns[-1]["role"] != "user":
        raise ValueError("SFT messages must end with a user message")
    return turns


def _answer_span(input_ids: list[int], start: int, eos_ids) -> tuple[int, int]:
    """[start, end) of the supervised answer: its tokens through the first EOS."""
    for position in range(start, len(input_ids)):
        if input_ids[position] in eos_ids:
            if position == start:
                raise ValueError("SFT answer must contain at least one token before EOS")
            return start, position + 1
    raise ValueError("completed SFT answer must contain a checkpoint EOS token")


def encode_example(record: dict, tokenizer: ModelTokenizer, *, max_length: int, enable_thinking: bool = False) -> dict:
    if not (type(max_length) is int and max_length >= 2):
        raise ValueError("max_length must be an integer of at least 2")
    turns = _conversation(record)
    prompt_ids, input_ids = tokenizer.encode_completion(turns, record["answer"],
                                                        chat_template_kwargs={"enable_thinking": enable_thinking})
    if len(input_ids) > max_length:
        raise ValueError(f"SFT example has {len(input_ids)} tokens, exceeding max_length={max_length}; "
                         "truncation is disabled")
    begin, end = _answer_span(input_ids, len(prompt_ids), tokenizer.eos_token_ids)
    labels = [IGNORE] * begin + input_ids[begin:end] + [IGNORE] * (len(input_ids) - end)
    return {"input_ids": input_ids, "labels": labels, "attention_mask": [1] * len(input_ids), "prompt_ids": prompt_ids}


def load_jsonl(path, tokenizer: ModelTokenizer, *, max_length: int, enable_thinking: bool = False) -> list[dict]:
    examples = []
    for number, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), start=1):
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
    """Right-padded [B, L] tensors; L is the longest example rounded up to the multiple."""
    if not examples:
        raise ValueError("cannot collate an empty SFT batch")
    if not (type(pad_token_id) is int and pad_token_id >= 0):
        raise ValueError("pad_token_id must be a nonnegative integer")
    if not (type(pad_to_multiple_of) is int and pad_to_multiple_of > 0):
        raise ValueError("pad_to_multiple_of must be a positive integer")
    for e in examples:
        size = len(e["input_ids"])
        if size == 0 or len(e["labels"]) != size or len(e["attention_mask"]) != size:
            raise ValueError("SFT input_ids, labels and attention_mask must have the same nonzero length")
    longest = max(len(e["input_ids"]) for e in examples)
    width = -(-longest // pad_to_multiple_of) * pad_to_multiple_of
    fill = {"input_ids": pad_token_id, "labels": IGNORE, "attention_mask": 0}
    return {name: torch.tensor([e[name] + [value] * (width - len(e[name])) for e in examples], dtype=torch.long)
            for name, value in fill.items()}


__all__ = ["collate_examples", "encode_example", "load_jsonl"]
