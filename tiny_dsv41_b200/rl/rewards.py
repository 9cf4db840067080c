"""Rewards computed on decoded response text, with strict parsers that never execute anything.

The rewards and what they accept are the contract of ``dsv41_train/rl/rewards.py`` (a run config
names them; the same prompt must score the same on either side). The expected answer is always
the record's ``metadata["answer"]``; a missing or unparsable expected answer is an error, while a
response that does not parse scores 0.

* ``text_exact_match`` - the final answer, NFKC-normalised with whitespace runs collapsed (case
  kept), equals the expected one treated the same way.
* ``numeric_answer`` - exact rational equality. Accepted forms: signed integers (optionally with
  thousands separators), decimals and scientific numbers (exponent magnitude <= 1000), ``a/b``,
  ``\\frac{a}{b}``, and a trailing ``%`` (divides by 100); at most 512 characters; a zero
  denominator does not parse.
* ``json_match`` - the response is one JSON value, or one fenced (json or unlabelled) code block
  holding one; no duplicate object keys; numbers compare as exact decimals and every value keeps
  its JSON type (true never equals 1); array order matters, object key order does not. The
  expected answer is the metadata value itself.

Final-answer extraction: a terminal ``<answer>...</answer>`` tag that is not nested in an open
tag is unwrapped; numeric answers may also come from a terminal, balanced ``\\boxed{...}`` or from
whatever follows the last ``####``. Prose without such a marker is never searched for numbers.
"""

from __future__ import annotations

import json
import math
import re
import unicodedata
from decimal import Decimal
from fractions import Fraction
from typing import Any, Callable

TEXT_REWARDS = {"text_exact_match", "numeric_answer", "json_match"}
_NUMBER = re.compile(r"[+-]?(?:(?:[0-9]+|[0-9]{1,3}(?:,[0-9]{3})+)(?:\.[0-9]*)?|\.[0-9]+)(?:[eE]([+-]?[0-9]+))?")
_LATEX_FRACTION = re.compile(r"\\frac\{([^{}]+)\}\{([^{}]+)\}")
_FENCE = re.compile(r"```(?:json)?[ \t]*\r?\n(.*?)\r?\n```", re.DOTALL)
_MAX_EXPONENT = 1000
_MAX_NUMERIC_CHARS = 512
_OPEN, _CLOSE, _BOXED = "<answer>", "</answer>", "\\boxed{"
_PARSE_ERRORS = (ValueError, ArithmeticError, RecursionError)


# -- locating the final answer --------------------------------------------------------------------
def _strip_answer_tag(text: str) -> str:
    if not text.endswith(_CLOSE):
        return text
    opening = text.rfind(_OPEN)
    before = text[:opening]
    if opening < 0 or before.rfind(_OPEN) > before.rfind(_CLOSE):
        return text  # unclosed or nested tags are not an answer
    return text[opening + len(_OPEN):-len(_CLOSE)].strip()


def _terminal_boxed(text: str) -> str | None:
    begin = text.rfind(_BOXED)
    if begin < 0:
        return None
    depth = 0
    for index in range(begin + len(_BOXED) - 1, len(text)):
        depth += {"{": 1, "}": -1}.get(text[index], 0)
        if depth == 0:
            return text[begin + len(_BOXED):index].strip() if index == len(text) - 1 else None
    return None


def final_answer(text: str, *, numeric: bool = False) -> str:
    answer = _strip_answer_tag(text.strip())
    if not numeric:
        return answer
    boxed = _terminal_boxed(answer)
    if boxed is not None:
        return boxed
    return answer.rsplit("####", 1)[1].strip() if "####" in answer else answer


# -- parsers ----------------------------------------------------------------------------------------
def parse_text(value: Any) -> str:
    if isinstance(value, str):
        normalised = " ".join(unicodedata.normalize("NFKC", final_answer(value)).split())
        if normalised:
            return normalised
    raise ValueError("expected a nonempty text answer")


def _rational(token: str) -> Fraction:
    token = token.strip()
    match = _NUMBER.fullmatch(token)
    if match is None:
        raise ValueError("expected a finite numeric scalar")
    exponent = match.group(1)
    if exponent is not None and abs(int(exponent)) > _MAX_EXPONENT:
        raise ValueError("numeric exponent magnitude exceeds 1000")
    return Fraction(Decimal(token.replace(",", "")))


def parse_number(value: Any) -> Fraction:
    if type(value) not in (str, int, float) or (type(value) is float and not math.isfinite(value)):
        raise ValueError("expected a finite numeric answer")
    text = final_answer(str(value), numeric=True)
    if len(text) > _MAX_NUMERIC_CHARS:
        raise ValueError("numeric answer exceeds 512 characters")
    scale = Fraction(1)
    if text.endswith("%"):
        text, scale = text[:-1].strip(), Fraction(1, 100)
    latex = _LATEX_FRACTION.fullmatch(text)
    parts = list(latex.groups()) if latex is not None else text.split("/")
    if len(parts) > 2:
        raise ValueError("expected a single scalar or fraction")
    number = _rational(parts[0])
    if len(parts) == 2:
        denominator = _rational(parts[1])
        if denominator == 0:
            raise ValueError("numeric answer has a zero denominator")
        number /= denominator
    return number * scale


def typed_json(value: Any, *, decoded: bool = False) -> Any:
    """A JSON value as (type tag, payload) pairs, numbers as exact finite decimals."""
    kind = type(value)
    if value is None or kind in (bool, str):
        return (kind.__name__, value)
    if kind in (int, float) or (decoded and kind is Decimal):
        number = Decimal(str(value))
        if not number.is_finite():
            raise ValueError("JSON numbers must be finite")
        return ("number", number)
    if isinstance(value, list):
        return ("array", [typed_json(item, decoded=decoded) for item in value])
    if isinstance(value, dict) and all(isinstance(key, str) for key in value):
        return ("object", {key: typed_json(item, decoded=decoded) for key, item in value.items()})
    raise ValueError("expected a JSON value with string object keys")


def _distinct_pairs(pairs):
    seen = set()
    for key, _ in pairs:
        if key in seen:
            raise ValueError("duplicate JSON object key")
        seen.add(key)
    return dict(pairs)


def parse_json(text: str) -> Any:
    body = text.strip()
    fenced = _FENCE.fullmatch(body)
    if fenced is not None:
        body = fenced.group(1)
    return typed_json(json.loads(body, object_pairs_hook=_distinct_pairs, parse_float=Decimal), decoded=True)


# -- rewards ----------------------------------------------------------------------------------------
# spec -> (parser of the expected metadata answer, parser of the decoded response)
_PARSERS: dict[str, tuple[Callable[[Any], Any], Callable[[str], Any]]] = {
    "text_exact_match": (parse_text, parse_text),
    "numeric_answer": (parse_number, parse_number),
    "json_match": (typed_json, parse_json),
}


def build_text_reward(spec: str, tokenizer):
    if spec not in _PARSERS:
        raise ValueError(f"unknown text reward {spec!r}")
    if not callable(getattr(tokenizer, "decode", None)):
        raise ValueError(f"reward {spec!r} requires a tokenizer with decode()")
    parse_expected, parse_response = _PARSERS[spec]

    def reward(record, response_ids) -> float:
        try:
            expected = parse_expected(record.metadata["answer"])
        except (KeyError, *_PARSE_ERRORS) as error:
            raise ValueError(f"reward {spec!r} requires valid metadata['answer']: {error}") from error
        try:
            text = tokenizer.decode(response_ids, skip_special_tokens=True)
        except ValueError:
            return 0.0
        if not isinstance(text, str):
            raise ValueError("tokenizer.decode() must return text")
        try:
            return float(parse_response(text) == expected)
        except _PARSE_ERRORS:
            return 0.0

    return reward


__all__ = ["TEXT_REWARDS", "build_text_reward", "final_answer", "parse_json", "parse_number", "parse_text",
           "typed_json"]
