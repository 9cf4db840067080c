"""Rollout contracts, coordinator (admission, quarantine), event store and the CLI run on CPU."""

import asyncio
import json
from pathlib import Path

import pytest

from tiny_dsv41_b200.rollout.contracts import (CancellationToken, EpisodeIdentity, EpisodePlan, EpisodeResult,
                                               ResourceRequirements, TaskSpec, request_uncertain)
from tiny_dsv41_b200.rollout.coordinator import Coordinator
from tiny_dsv41_b200.rollout.events import EventStore

MODEL = Path(__file__).resolve().parents[1] / "examples" / "tiny-dsv41"


class _Echo:
    def __init__(self, uncertain_for=()):
        self.active = self.peak = 0
        self.uncertain_for = set(uncertain_for)

    async def execute(self, plan, cancellation):
        self.active += 1
        self.peak = max(self.peak, self.active)
        await asyncio.sleep(0.01)
        self.active -= 1
        state = {"state": "unknown"} if plan.identity.sample_index in self.uncertain_for else None
        return EpisodeResult(plan.identity, "completed", "verified", True, "clean",
                             {"sample": plan.identity.sample_index}, None, request_state=state)


def _plans(groups=2, size=3):
    task = lambda i: TaskSpec("prompt-response", f"t{i}", "0" * 64, {"prompt_response": {}},
                              ResourceRequirements("cpu"))
    return [EpisodePlan(EpisodeIdentity("run", "prompt-response", f"t{g}", str(g), s), task(g))
            for g in range(groups) for s in range(size)]


def test_contract_rules():
    with pytest.raises(ValueError):
        TaskSpec("unknown", "t", "x", {}, ResourceRequirements("cpu"))
    with pytest.raises(ValueError):
        ResourceRequirements("cpu", cpu=-1)
    assert request_uncertain({"delivery": {"state": "Unknown outcome"}})
    assert not request_uncertain({"state": "completed"})
    token = CancellationToken()
    token.cancel("first")
    token.cancel("second")
    assert token.cancelled() and token.reason == "first"


def test_coordinator_limits_events_and_quarantine(tmp_path):
    backend = _Echo(uncertain_for={2})
    store = EventStore(tmp_path / "events", "run")
    coordinator = Coordinator({"prompt-response": backend}, max_workers=3, max_groups=2, event_store=store)
    results = asyncio.run(coordinator.run_wave(_plans()))
    assert [r.native_outcome["sample"] for r in results] == [0, 1, 2, 0, 1, 2]
    assert backend.peak <= 3 and coordinator.quarantined == 2
    assert coordinator.usable_workers == 1
    stuck = Coordinator({"prompt-response": _Echo(uncertain_for={0})}, max_workers=1)
    with pytest.raises(RuntimeError):  # the only slot is quarantined by the first episode
        asyncio.run(stuck.run_wave(_plans(1, 2)))
    store.close()
    events = [json.loads(line)["event"] for line in (tmp_path / "events" / "events.jsonl").read_text().splitlines()]
    assert events.count("finished") == 6 and events.count("quarantined") == 2
    assert len(list((tmp_path / "events" / "results").iterdir())) == 6


def test_cli_run(tmp_path, capsys):
    from tiny_dsv41_b200.rollout.cli import main

    tasks = tmp_path / "tasks.jsonl"
    tasks.write_text("\n".join(json.dumps({"prompt_ids": [1, 3, 9 + i, 6, 4], "target_ids": [9, 10]}) for i in range(2)))
    main(["inspect", "--tasks", str(tasks)])
    assert json.loads(capsys.readouterr().out)["tasks"] == 2
    main(["run", "--tasks", str(tasks), "--model-dir", str(MODEL), "--output-dir", str(tmp_path / "out"),
          "--random-init", "--group-size", "2", "--max-new-tokens", "2"])
    summary = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert summary["episodes"] == 4 and summary["eligible"] == 4
    assert (tmp_path / "out" / "summary.json").is_file()


class _Lifecycle(_Echo):
    def __init__(self, **kw):
        super().__init__(**kw)
        self.starts = self.closes = 0

    async def start(self):
        self.starts += 1

    async def close(self):
        self.closes += 1


def test_persistent_stream_session():
    backend = _Lifecycle()

    async def scenario():
        coord = Coordinator({"prompt-response": backend}, max_workers=2, max_groups=1)
        await coord.open_stream(max_pending=3)
        plans = _plans(groups=3, size=3)
        first = await coord.execute_stream_group(plans[0:3], sequence=0)
        assert [r.identity.sample_index for r in first] == [0, 1, 2]
        with pytest.raises(ValueError):  # a replayed sequence number
            await coord.execute_stream_group(plans[3:6], sequence=0)
        with pytest.raises(ValueError):  # two groups at once
            await coord.execute_stream_group(plans[2:5], sequence=5)
        with pytest.raises(ValueError):  # more pending episodes than the credit
            await coord.execute_stream_group(plans[3:6] + [plans[6]], sequence=6)
        await coord.execute_stream_group(plans[3:6], sequence=7)
        await coord.pause_stream()
        with pytest.raises(ValueError):  # paused: no admission
            await coord.execute_stream_group(plans[6:9], sequence=8)
        coord.resume_stream()
        await coord.execute_stream_group(plans[6:9], sequence=9)
        await coord.close_stream()
        return coord

    coord = asyncio.run(scenario())
    assert backend.starts == 1 and backend.closes == 1
    assert backend.peak <= 2 and coord.quarantined == 0


def test_stream_stops_after_uncertain_request():
    backend = _Lifecycle(uncertain_for={1})

    async def scenario():
        coord = Coordinator({"prompt-response": backend}, max_workers=3)
        await coord.open_stream(max_pending=3)
        plans = _plans(groups=2, size=3)
        await coord.execute_stream_group(plans[:3], sequence=1)
        with pytest.raises(ValueError):
            await coord.execute_stream_group(plans[3:], sequence=2)
        with pytest.raises(RuntimeError):
            coord.resume_stream()
        await coord.close_stream()
        return coord

    coord = asyncio.run(scenario())
    assert coord.quarantined == 1
