"""Benchmark episodes assembled into GRPO training groups (rollout/benchmark_training.py)."""

import hashlib

import pytest

from tiny_dsv41_b200.rollout import benchmark_training as B
from tiny_dsv41_b200.rollout import contracts as C
from tiny_dsv41_b200.rollout import training as T

SHA = T.token_digest([1, 2])  # the initial context of every sampled turn below
SRC = hashlib.sha256(b"source").hexdigest()
POLICY = T.PolicyRef(2, hashlib.sha256(b"p").hexdigest(), "run")


def _plans(group="g0", size=2):
    task = C.TaskSpec("kernelbench", "level1/7", SRC, {"native_case": {"id": 7}}, C.ResourceRequirements("gpu"))
    return [C.EpisodePlan(C.EpisodeIdentity("run", "kernelbench", "level1/7", group, i), task) for i in range(size)]


def _result(plan, correct=True, request_ok=True):
    turn = T.TurnTrace(1, f"req-{plan.identity.sample_index}", [1, 2], [3], [-0.5], POLICY, "eos", 1)
    state = "response_received" if request_ok else "sent"
    return C.EpisodeResult(plan.identity, "completed", "passed" if correct else "failed", True, "verified",
                           {"final_correct": correct, "training_turns": [turn.to_dict()]}, {"log": "x"},
                           request_state={"requests": {turn.request_id: {"state": state,
                                                                          "training_evidence": "validated"}}},
                           source_sha256=SRC)


def _registration(group_id=0, plans=None):
    return B.GroupRegistration(group_id, plans or _plans(), POLICY, SHA, SHA,
                               B.RewardPolicy("kernelbench", "native-final-correctness-v1"))


def test_group_completes_with_rewards():
    assembler = B.GroupAssembler(max_groups=1, max_episodes=4)
    plans = _plans()
    assembler.register(_registration(0, plans))
    assert assembler.complete(_result(plans[1], correct=False)) is None
    group = assembler.complete(_result(plans[0], correct=True))
    assert isinstance(group, T.TrainingGroup)
    assert [s.reward for s in group.samples] == [1.0, 0.0]
    assert group.samples[0].evidence["reward_mapping"] == "native-final-correctness-v1"
    T.loads(T.dumps(group))  # a valid, serialisable training record
    # the group is gone: its episodes cannot complete twice, a new monotonic group can register
    with pytest.raises(ValueError):
        assembler.complete(_result(plans[0]))
    assembler.register(_registration(1, _plans("g1")))


def test_unverified_request_excludes_the_group():
    assembler = B.GroupAssembler()
    plans = _plans()
    assembler.register(_registration(0, plans))
    assembler.complete(_result(plans[0]))
    excluded = assembler.complete(_result(plans[1], request_ok=False))
    assert isinstance(excluded, B.GroupExclusion)
    assert excluded.reasons[0].startswith("sample-1") and excluded.to_dict()["kind"] == "excluded_training_group"


def test_registration_rules_and_capacity():
    with pytest.raises(ValueError):
        B.RewardPolicy("kernelbench", "terminal-validated-verifier-v1")
    with pytest.raises(ValueError):
        _registration(plans=_plans(size=1))
    assembler = B.GroupAssembler(max_groups=1, max_episodes=4)
    assembler.register(_registration(3))
    with pytest.raises(ValueError):  # capacity: one open group
        assembler.register(_registration(4, _plans("g4")))
    with pytest.raises(ValueError):  # ids must grow
        B.GroupAssembler().register(_registration(-1))


def test_artifact_policy_hashes_the_run_identity():
    artifact = {"version": 2, "digest": POLICY.digest, "lineage": "run", "identity": {"config": "abc"},
                "sampling": {"temperature": 1.0, "top_p": 1, "top_k": 0}}
    ref = B.artifact_policy(artifact, identities={"tokenizer_sha256": SHA})
    assert ref.identities["tokenizer_sha256"] == SHA and len(ref.identities["run_identity_sha256"]) == 64
