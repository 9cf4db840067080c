"""Example scripts shipped beside the framework."""

import importlib.util
import json
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _load(path):
    spec = importlib.util.spec_from_file_location(path.stem, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_prepare_identity_sft(tmp_path):
    script = _load(ROOT / "examples" / "sft" / "prepare_identity_sft.py")
    script.main(["--model-path", str(ROOT / "examples" / "tiny-dsv41"), "--output-dir", str(tmp_path),
                 "--min-active-tokens", "120", "--max-length", "300", "--diverse-training", "--answer-suffix", " <eos>"])
    train = [json.loads(line) for line in (tmp_path / "train.jsonl").read_text().splitlines()]
    evaluation = [json.loads(line) for line in (tmp_path / "eval.jsonl").read_text().splitlines()]
    lengths = json.loads((tmp_path / "lengths.json").read_text())
    assert len(train) == 32 and len(evaluation) == 5
    assert sum(n >= 120 for n in lengths["train"]) == 16  # the long half of the diverse set
    assert all(script.IDENTITY not in row["prompt"] for row in train + evaluation)
    trained = {row["prompt"].rsplit(": ", 1)[-1] for row in train} | {row["prompt"] for row in train}
    assert not any(q in trained for q in script.EVAL_QUESTIONS)
