"""Write a long-context identity SFT set: training rows whose final question asks for the model's
name after a long neutral background, and fixed evaluation prompts that are never trained on.

Same role as ``scripts/prepare_identity_sft.py`` of the reference (long authored QA to check that
SFT reaches the answer through thousands of context tokens); the questions, the background text and
the default identity here are this file's own.

    python examples/sft/prepare_identity_sft.py --model-path <checkpoint with tokenizer.json> \
        --output-dir data/identity [--min-active-tokens 4096 --max-length 4608] \
        [--include-short-training | --diverse-training]

Outputs ``train.jsonl`` and ``eval.jsonl`` (``{"prompt", "answer"}`` records, the format
``python -m tiny_dsv41_b200.train.sft`` reads) and ``lengths.json`` (encoded token counts).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from tiny_dsv41_b200.rl.tokenizer import ModelTokenizer  # noqa: E402
from tiny_dsv41_b200.train.sft_data import encode_example  # noqa: E402

IDENTITY = "Tiny-DSV41 on B200"
TRAIN_QUESTIONS = ("Who are you?", "What is your name?", "Please introduce yourself.", "Which model are you?")
EVAL_QUESTIONS = ("How should I address the assistant answering me?", "Tell me the name of this assistant.",
                  "Which model is producing these replies?", "Who am I talking to?",
                  "State the name you go by, nothing else.")
BACKGROUND = (
    "The harbour log lists each ferry departure with its berth number and the weather at sailing time.",
    "A weather station notes wind speed, humidity and cloud cover every hour, leaving gaps blank.",
    "The workshop sorts brass fittings by thread size and records which drawer each batch went into.",
    "A hiking club marks trail junctions with numbered posts and checks the signs after each storm.",
)
HELD_OUT_BACKGROUND = ("An orchard survey counts blossoms per branch and records the date of the first frost.",)
DIVERSE_QUESTIONS = (
    "For the service check, print the official identifier of the current assistant.",
    "Sign this conversation with your model name only.",
    "First time here: which model am I using? Answer with the name alone.",
    "The lab sheet has a field 'model used'. What goes in it?",
    "Fill in the 'model' column of the report with your own name.",
    "Output your model identifier without any preamble.",
    "If you had a name badge, what would it say?",
    "Give me the assistant's model name for my records.",
)
DIVERSE_BACKGROUNDS = (
    ("A bakery weighs every batch of dough and logs the oven temperature for each tray.",
     "Flour sacks are counted at closing time and the empty ones stacked by the door."),
    ("The bus depot inspects seats, lights and route boards, dating each completed checklist.",
     "Bulbs that failed the test are listed on the handover sheet for the night crew."),
    ("A seed bank files samples by collection site and labels each jar with its shelf code.",
     "Germination trials record sprout length weekly; unchanged samples keep their old labels."),
    ("River samplers seal every bottle, noting the site and the minute it was filled.",
     "After rinsing, the bench instruments are ticked off against the inventory list."),
)


def long_example(tokenizer, question, *, min_tokens, max_tokens, sentences=BACKGROUND, answer=IDENTITY):
    """Prepend numbered background lines until the encoded example reaches ``min_tokens``."""
    lines = []
    while True:
        lines.append(f"Note {len(lines) + 1}: {sentences[len(lines) % len(sentences)]}")
        prompt = "Background notes follow.\n" + "\n".join(lines) + "\nNow answer the final question: " + question
        record = {"prompt": prompt, "answer": answer}
        if IDENTITY in prompt:
            raise ValueError("the identity answer leaked into a prompt")
        encoded = encode_example(record, tokenizer, max_length=max_tokens)  # raises once too long
        if len(encoded["input_ids"]) >= min_tokens:
            return record, len(encoded["input_ids"])


def short_example(tokenizer, question, *, max_tokens, answer=IDENTITY):
    record = {"prompt": question, "answer": answer}
    return record, len(encode_example(record, tokenizer, max_length=max_tokens)["input_ids"])


def build(tokenizer, *, min_tokens, max_tokens, include_short=False, diverse=False, answer=IDENTITY):
    train, lengths = [], []
    kw = {"max_tokens": max_tokens, "answer": answer}
    if diverse:  # four blocks of four long and four short rows
        for block, sentences in enumerate(DIVERSE_BACKGROUNDS):
            questions = DIVERSE_QUESTIONS[(2 * block) % len(DIVERSE_QUESTIONS):][:2] + TRAIN_QUESTIONS[:2]
            for q in questions:
                rec, n = long_example(tokenizer, q, min_tokens=min_tokens, sentences=sentences, **kw)
                train.append(rec), lengths.append(n)
            for q in questions:
                rec, n = short_example(tokenizer, q, **kw)
                train.append(rec), lengths.append(n)
    else:
        for q in TRAIN_QUESTIONS:
            rec, n = long_example(tokenizer, q, min_tokens=min_tokens, **kw)
            train.append(rec), lengths.append(n)
        if include_short:
            for q in TRAIN_QUESTIONS:
                rec, n = short_example(tokenizer, q, **kw)
                train.append(rec), lengths.append(n)
    evaluation, eval_lengths = [], []
    for i, q in enumerate(EVAL_QUESTIONS):
        if i < 3:  # unseen question after an unseen background
            rec, n = long_example(tokenizer, q, min_tokens=min_tokens, sentences=HELD_OUT_BACKGROUND, **kw)
        else:
            rec, n = short_example(tokenizer, q, **kw)
        evaluation.append(rec), eval_lengths.append(n)
    return train, evaluation, {"train": lengths, "eval": eval_lengths}


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--model-path", required=True, help="directory with tokenizer.json / tokenizer_config.json")
    parser.add_argument("--output-dir", required=True)
    parser.add_argument("--min-active-tokens", type=int, default=4096, help="minimum tokens of each long example")
    parser.add_argument("--max-length", type=int, default=4608)
    parser.add_argument("--answer-suffix", default="",
                        help="text appended to the answer, e.g. ' <eos>' for chat templates that do not close the "
                             "assistant turn with an EOS token")
    group = parser.add_mutually_exclusive_group()
    group.add_argument("--include-short-training", action="store_true", help="also train on the bare questions")
    group.add_argument("--diverse-training", action="store_true",
                       help="32 rows: four blocks of four long and four short examples")
    args = parser.parse_args(argv)
    if not 2 <= args.min_active_tokens < args.max_length:
        parser.error("require 2 <= --min-active-tokens < --max-length (room for the final question and answer)")
    tokenizer = ModelTokenizer(args.model_path)
    train, evaluation, lengths = build(tokenizer, min_tokens=args.min_active_tokens, max_tokens=args.max_length,
                                       include_short=args.include_short_training, diverse=args.diverse_training,
                                       answer=IDENTITY + args.answer_suffix)
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    for name, rows in (("train.jsonl", train), ("eval.jsonl", evaluation)):
        with open(out / name, "w", encoding="utf-8") as f:
            for row in rows:
                f.write(json.dumps(row, ensure_ascii=False) + "\n")
    (out / "lengths.json").write_text(json.dumps(lengths, indent=1))
    print(json.dumps({"train_rows": len(train), "eval_rows": len(evaluation), "min_train_tokens": min(lengths["train"]),
                      "max_train_tokens": max(lengths["train"])}))


if __name__ == "__main__":
    main()
