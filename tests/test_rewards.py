"""Text rewards: the parsers accept and reject exactly what the reference's do (differential check
on a fixed set of answers when the reference package is installed), plus fixed expectations."""

from fractions import Fraction
from types import SimpleNamespace

import pytest

from tests.ref_oracle import import_reference, reference_available
from tiny_dsv41_b200.rl import rewards as R

CASES = ["42", "  The answer is \\boxed{3/4}", "x #### 1,234.5", "<answer>12%</answer>", "\\frac{1}{3}", "1e1001",
         "abc", "$5.", "<answer><answer>7</answer>", "\\boxed{\\frac{2}{4}}", '{"a": 1}', '{"a":1,"a":2}', "NaN",
         "3/0", "1,23", "```json\n[1, 2.0, true]\n```", "1/2/3", 5, 2.5, float("nan"), "x" * 600, "[1e400]",
         "-.5e-3", "\\boxed{1} trailing", "<answer> 3 </answer>", "1,234,567.00"]


def _outcome(fn, value):
    try:
        return "ok", fn(value)
    except Exception as error:  # noqa: BLE001 - the exception type is what is compared
        return "error", type(error).__name__


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_parsers_match_the_reference():
    import_reference()
    from dsv41_train.rl import rewards as ref

    pairs = ((ref._numeric_answer, R.parse_number), (ref._text_answer, R.parse_text),
             (ref._json_answer, R.parse_json), (ref._json_value, R.typed_json))
    for value in CASES:
        for theirs, ours in pairs:
            assert _outcome(ours, value) == _outcome(theirs, value), (value, ours.__name__)


def test_numeric_forms_and_json_types():
    assert R.parse_number("<answer>50%</answer>") == Fraction(1, 2) == R.parse_number("\\frac{1}{2}")
    assert R.parse_number("so #### 1,000") == 1000
    with pytest.raises(ValueError):
        R.parse_number("3/0")
    assert R.parse_json("[true]") != R.parse_json("[1]")
    assert R.parse_json('{"b": 1, "a": 2.50}') == R.typed_json({"a": 2.5, "b": 1})


def test_text_reward_scores_and_requires_an_answer():
    tokenizer = SimpleNamespace(decode=lambda ids, skip_special_tokens=True: "".join(map(str, ids)))
    reward = R.build_text_reward("numeric_answer", tokenizer)
    record = SimpleNamespace(metadata={"answer": "12"}, target_ids=None)
    assert reward(record, [1, 2]) == 1.0 and reward(record, [1, 3]) == 0.0
    with pytest.raises(ValueError):
        reward(SimpleNamespace(metadata={}, target_ids=[1]), [1])
