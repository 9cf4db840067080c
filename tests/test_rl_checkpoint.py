"""RL checkpoint formats: atomic save, digest-named policy artifacts, acknowledgements, resume identity."""

import json

import pytest
import torch

from tiny_dsv41_b200.rl import checkpoint as ck
from tiny_dsv41_b200.utils.stage_timings import StageTimings


class _Policy(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(4, 4)
        self.b = torch.nn.Linear(4, 2)

    def trainable_state_dict(self):
        return {k: v.detach().clone() for k, v in self.a.state_dict().items()}

    def frozen_state_dict(self):
        return {k: v.detach().clone() for k, v in self.b.state_dict().items()}

    def load_trainable_state_dict(self, s):
        self.a.load_state_dict(s)

    def load_frozen_state_dict(self, s):
        self.b.load_state_dict(s)


def test_policy_artifact_roundtrip(tmp_path):
    torch.manual_seed(0)
    src, dst = _Policy(), _Policy()
    art = ck.publish_policy_artifact(src, 3, tmp_path / "policies", lineage="run-a", identity={"x": 1},
                                     sampling={"temperature": 1.0})
    assert art["path"].endswith(f"policy-00000003-{art['digest']}.pt")
    ack = ck.load_policy_artifact(dst, art)
    ck.validate_policy_ack(ack, art)
    for (k, p), q in zip(src.state_dict().items(), dst.state_dict().values()):
        assert torch.equal(p, q), k
    again = ck.publish_policy_artifact(src, 3, tmp_path / "policies", lineage="run-a", identity={"x": 1},
                                       sampling={"temperature": 1.0})
    assert again["digest"] == art["digest"]
    with pytest.raises(RuntimeError):
        ck.validate_policy_ack({**ack, "version": 4}, art)
    bad = dict(art, lineage="run-b")
    with pytest.raises(ValueError):
        ck.load_policy_artifact(dst, bad)


def test_digest_mismatch_rejected(tmp_path):
    art = ck.publish_policy_artifact(_Policy(), 0, tmp_path, lineage="r", identity={}, sampling={})
    with pytest.raises(ValueError):
        ck.load_policy_artifact(_Policy(), dict(art, digest="0" * 64))


def test_atomic_save_and_identity(tmp_path):
    ck.atomic_save({"a": torch.ones(2)}, tmp_path / "x.pt")
    assert torch.equal(torch.load(tmp_path / "x.pt")["a"], torch.ones(2))
    assert [p.name for p in tmp_path.iterdir()] == ["x.pt"]
    model = tmp_path / "m"
    model.mkdir()
    (model / "config.json").write_text("{}")
    (model / "tokenizer.json").write_text("{}")
    data = tmp_path / "d.jsonl"
    data.write_text('{"prompt": "1+1", "answer": "2"}\n')
    a = ck.run_identity(model, data, True)
    ck.validate_identity(a, ck.run_identity(model, data, True))
    data.write_text('{"prompt": "1+2", "answer": "3"}\n')
    with pytest.raises(ValueError):
        ck.validate_identity(a, ck.run_identity(model, data, True))


def test_stage_timings(tmp_path):
    t = StageTimings(tmp_path / "t.jsonl")
    with t.interval("rollout", group=1):
        pass
    assert t.call("train", lambda x: x + 1, 1) == 2
    rows = [json.loads(line) for line in (tmp_path / "t.jsonl").read_text().splitlines()]
    assert [r["stage"] for r in rows] == ["rollout", "train"]
    assert rows[0]["details"] == {"group": 1} and rows[0]["seconds"] >= 0
