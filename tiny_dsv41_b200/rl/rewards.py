"""Decoded-text rewards with strict, non-executing parsers: ``text_exact_match`` (NFKC,
whitespace-collapsed final answer), ``numeric_answer`` (exact rational comparison of a terminal
answer tag, ``\\boxed{}``, ``####`` marker, decimal/scientific/fraction/percent forms) and
``json_match`` (duplicate-key-free JSON equality). Same contract as ``dsv41_train/rl/rewards.py``."""

from __future__ import annotations

import json
import re
import unicodedata
from decimal import Decimal, InvalidOperation
from fractions import Fraction
from typing import Any

TEXT_REWARDS = {"text_exact_match", "numeric_answer", "json_match"}
_NUMBER = re.compile(r"[+-]?(?:(?:[0-9]+|[0-9]{1,3}(?:,[0-9]{3})+)(?:\.[0-9]*)?|\.[0-9]+)(?:[eE]([+-]?[0-9]+))?")
_FRAC = re.compile(r"\\frac\{([^{}]+)\}\{([^{}]+)\}")


def _final_answer(text: str, *, numeric: bool = False) -> str:
    text = text.strip()
    if text.endswith("</answer>"):
        start = text.rfind("<answer>")
        prefix = text[:start]
        if start >= 0 and prefix.rfind("<answer>") <= prefix.rfind("</answer>"):
            text = text[start + len("<answer>"):-len("</answer>")].strip()
    if not numeric:
        return text
    start = text.rfind("\\boxed{")
    if start >= 0:
        content = start + len("\\boxed{")
        depth = 1
        for i in range(content, len(text)):
            if text[i] == "{":
                depth += 1
            elif text[i] == "}":
                depth -= 1
                if depth == 0:
                    if i == len(text) - 1:
                        return text[content:i].strip()
                    break
    if "####" in text:
        return text.rsplit("####", 1)[1].strip()
    return text


def _text_answer(value: Any) -> str:
    if not isinstance(value, str):
        raise ValueError("expected a nonempty text answer")
    answer = " ".join(unicodedata.normalize("NFKC", _final_answer(value)).split())
    if not answer:
        raise ValueError("expected a nonempty text answer")
    return answer


def _decimal(text: str) -> Fraction:
    match = _NUMBER.fullmatch(text.strip())
    if match is None:
        raise ValueError("expected a finite numeric scalar")
    if match.group(1) is not None and abs(int(match.group(1))) > 1000:
        raise ValueError("numeric exponent magnitude exceeds 1000")
    try:
        return Fraction(Decimal(text.strip().replace(",", "")))
    except (InvalidOperation, ValueError) as error:
        raise ValueError("expected a finite numeric scalar") from error


def _numeric_answer(value: Any) -> Fraction:
    if isinstance(value, (int, float)) and not isinstance(value, bool):
        return Fraction(Decimal(str(value)))
    if not isinstance(value, str):
        raise ValueError("expected a numeric answer")
    text = unicodedata.normalize("NFKC", _final_answer(value, numeric=True)).strip().rstrip(".")
    text = text.replace("$", "").strip()
    percent = text.endswith("%")
    if percent:
        text = text[:-1].strip()
    frac = _FRAC.fullmatch(text)
    if frac:
        result = _decimal(frac.group(1)) / _decimal(frac.group(2))
    elif text.count("/") == 1:
        a, b = text.split("/")
        result = _decimal(a) / _decimal(b)
    else:
        result = _decimal(text)
    return result / 100 if percent else result


def _unique_object(pairs):
    keys = [k for k, _ in pairs]
    if len(keys) != len(set(keys)):
        raise ValueError("duplicate JSON object key")
    return dict(pairs)


def _json_answer(text: str) -> Any:
    return json.loads(_final_answer(text), object_pairs_hook=_unique_object,
                      parse_constant=lambda c: (_ for _ in ()).throw(ValueError(c)))


def build_text_reward(spec: str, tokenizer):
    def reference(record):
        for key in ("answer", "target", "reference"):
            if key in record.metadata:
                return record.metadata[key]
        if record.target_ids is not None:
            return tokenizer.decode(record.target_ids)
        raise ValueError("text rewards require an answer in the record")

    def reward(record, response_ids):
        text = tokenizer.decode(response_ids)
        try:
            if spec == "text_exact_match":
                return float(_text_answer(text) == _text_answer(reference(record)))
            if spec == "numeric_answer":
                return float(_numeric_answer(text) == _numeric_answer(reference(record)))
            expected = reference(record)
            expected = _json_answer(expected) if isinstance(expected, str) else expected
            return float(_json_answer(text) == expected)
        except (ValueError, ZeroDivisionError, json.JSONDecodeError):
            return 0.0

    return reward


__all__ = ["TEXT_REWARDS", "build_text_reward"]
