"""GSM8K prompt selection with numeric rewards (``dsv41_train/rl/gsm8k.py:12-95``).

Only the official release files are accepted: the pinned revision and the SHA256 of each split
identify them (these identifiers must equal the reference's to select the same data). Selection
is a seeded shuffle that skips prompts longer than the token limit (no truncation); the reward
is the exact-rational ``numeric_answer``; the provenance record lists every selected id.
"""

from __future__ import annotations

import hashlib
import json
import random
from pathlib import Path

from .data import PromptRecord, build_reward
from .rewards import parse_number

DATASET_REVISION = "3101c7d5072418e28b9008a6636bde82a006892c"
SPLIT_SHA256 = {"train": "17f347dc51477c50d4efb83959dbb7c56297aba886e5544ee2aaed3024813465",
                "test": "3730d312f6e3440559ace48831e51066acaca737f6eabec99bccb9e4b3c39d14"}
SPLIT_SIZE = {"train": 7473, "test": 1319}
INSTRUCTION = "\nSolve the problem. End your answer with #### followed by the final numeric answer."


def load_split(path, split: str):
    if split not in SPLIT_SIZE:
        raise ValueError("GSM8K split must be train or test")
    path = Path(path)
    rows = []
    for index, line in enumerate(path.read_text().splitlines()):
        row = json.loads(line)
        if (not isinstance(row, dict) or not isinstance(row.get("question"), str) or not row["question"].strip()
                or not isinstance(row.get("answer"), str) or "####" not in row["answer"]):
            raise ValueError(f"{path}:{index + 1}: not an official GSM8K question/answer record")
        answer = row["answer"].rsplit("####", 1)[1].strip()
        parse_number(answer)  # a malformed reference answer aborts instead of scoring zero
        rows.append({"id": f"gsm8k:{split}:{index}", "question": row["question"], "answer": answer})
    if len(rows) != SPLIT_SIZE[split] or len({r["question"] for r in rows}) != len(rows):
        raise ValueError(f"official GSM8K {split} must contain {SPLIT_SIZE[split]} distinct questions")
    return rows, hashlib.sha256(path.read_bytes()).hexdigest()


def select_records(train, test, tokenizer, *, revision=DATASET_REVISION, seed=42, max_prompt_tokens=256,
                   max_train_groups=64, eval_questions=128):
    """Seeded, length-filtered selection from already loaded rows."""
    rng = random.Random(seed)
    train, test = list(train), list(test)
    rng.shuffle(train)
    rng.shuffle(test)
    selected, excluded = {}, {}
    for split, rows, count in (("train", train, max_train_groups), ("test", test, eval_questions)):
        selected[split], excluded[split] = [], []
        for row in rows:
            record = PromptRecord(tokenizer.encode_prompt(prompt=row["question"] + INSTRUCTION),
                                  metadata={**row, "dataset": "gsm8k", "split": split, "revision": revision})
            if len(record.prompt_ids) > max_prompt_tokens:
                excluded[split].append(row["id"])
                continue
            selected[split].append(record)
            if len(selected[split]) == count:
                break
        if len(selected[split]) != count:
            raise ValueError(f"not enough GSM8K {split} records fit the prompt limit")
    return selected, excluded


def prepare_data(train_path, test_path, tokenizer, *, revision, seed=42, max_prompt_tokens=256, max_train_groups=64,
                 eval_questions=128):
    if revision != DATASET_REVISION:
        raise ValueError("GSM8K revision differs from the pinned official dataset")
    if not 1 <= eval_questions <= SPLIT_SIZE["test"] or max_train_groups < 1 or max_prompt_tokens < 1:
        raise ValueError("use a nonempty held-out subset and train groups, with a positive prompt limit")
    train, train_hash = load_split(train_path, "train")
    test, test_hash = load_split(test_path, "test")
    if {"train": train_hash, "test": test_hash} != SPLIT_SHA256:
        raise ValueError("official GSM8K files differ from the pinned revision hashes")
    if {r["question"] for r in train} & {r["question"] for r in test}:
        raise ValueError("GSM8K training/test question overlap")
    selected, excluded = select_records(train, test, tokenizer, revision=revision, seed=seed,
                                        max_prompt_tokens=max_prompt_tokens, max_train_groups=max_train_groups,
                                        eval_questions=eval_questions)
    provenance = {"repository": "https://github.com/openai/grade-school-math", "revision": revision,
                  "train_sha256": train_hash, "test_sha256": test_hash, "seed": seed,
                  "max_prompt_tokens": max_prompt_tokens,
                  "selection": "seeded shuffle, exclude overlength prompts without truncation",
                  "subset_ids": {k: [r.metadata["id"] for r in v] for k, v in selected.items()},
                  "overlength_ids_encountered": excluded,
                  "reward": "numeric_answer: exact rational scalar after the final ####/box/answer tag; malformed output "
                            "scores zero",
                  "format_metric": "terminal #### marker followed by a valid numeric scalar; not part of reward"}
    return selected["train"], selected["test"], build_reward("numeric_answer", tokenizer=tokenizer), provenance


def formatting_correct(text: str) -> bool:
    if "####" not in text:
        return False
    try:
        parse_number(text.rsplit("####", 1)[1].strip())
        return True
    except (ValueError, ArithmeticError):
        return False


def wilson_interval(correct: int, total: int) -> list[float]:
    """95% Wilson score interval for a binomial proportion."""
    if total < 1 or not 0 <= correct <= total:
        raise ValueError("invalid binomial counts")
    z = 1.959963984540054  # standard normal 97.5% quantile
    p, z2 = correct / total, z * z
    center = (p + z2 / (2 * total)) / (1 + z2 / total)
    radius = z * ((p * (1 - p) / total + z2 / (4 * total ** 2)) ** 0.5) / (1 + z2 / total)
    return [center - radius, center + radius]


__all__ = ["DATASET_REVISION", "SPLIT_SHA256", "formatting_correct", "load_split", "prepare_data", "select_records",
           "wilson_interval"]
