"""Sealed Engram baselines, private role views and cumulative row deltas (CPU)."""

import os
import pickle
from pathlib import Path

import pytest
import torch

from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config
from tiny_dsv41_b200.rl.engram_state import EngramBaseline, EngramState, memfd_seals

MODEL = Path(__file__).resolve().parents[1] / "examples" / "tiny-dsv41"


def test_baseline_views_and_deltas():
    cfg = DeepSeekV41Config.from_json(MODEL / "config.json")
    base = EngramBaseline.create(MODEL, cfg, torch.float32, True, 7)
    name = next(iter(base.shapes))
    assert memfd_seals(base._fds[name]) & 8  # write-sealed
    learner, actor = EngramState(base, "learner", True), EngramState(base, "actor", False)
    before = actor.tables[name].weight.detach().clone()
    w = learner.tables[name].weight
    idx = torch.tensor([3, 9, 3])
    w.grad = torch.sparse_coo_tensor(idx[None], torch.ones(3, w.shape[1]), w.shape)
    with torch.no_grad():
        w[3] += 1.0
        w[9] -= 2.0
    learner.mark_touched()
    delta = learner.state_dict()
    assert delta["tables"][name]["indices"].tolist() == [3, 9]
    assert torch.equal(actor.tables[name].weight, before)  # private copy-on-write pages
    actor.load_state_dict(delta)
    assert torch.equal(actor.tables[name].weight[3], w[3].detach())
    empty = {**delta, "tables": {n: {"indices": torch.empty(0, dtype=torch.long),
                                     "values": torch.empty(0, base.shapes[n][1])} for n in base.shapes}}
    actor.load_state_dict(empty)  # back to the baseline rows
    assert torch.equal(actor.tables[name].weight, before)
    copy = pickle.loads(pickle.dumps(base))  # descriptors, not tensor storage, cross processes
    assert torch.equal(copy.view(name), base.view(name))
    with pytest.raises(ValueError):
        EngramState(base, "reference", False).load_state_dict(delta)
