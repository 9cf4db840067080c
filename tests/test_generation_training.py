"""Fail-closed training evidence from a generation route (rollout/generation_training.py)."""

import hashlib

import pytest

from tests.ref_oracle import import_reference, reference_available
from tiny_dsv41_b200.rollout import generation_training as G
from tiny_dsv41_b200.rollout import training as T

SHA = hashlib.sha256(b"x").hexdigest()


def _policy():
    return T.PolicyRef(4, hashlib.sha256(b"policy").hexdigest(), "run",
                       {"tokenizer_sha256": SHA, "chat_template_sha256": SHA}, {"temperature": 0.8, "top_p": 1,
                                                                                  "top_k": 0})


def _capabilities(policy):
    return {"schema_version": 1, **{name: True for name in G.TrainingGenerationContract.REQUIRED},
            "logprob_convention": "sampled_distribution", "policy": policy.to_dict()}


def _exchange(policy, request_id="req-1"):
    payload = {"model": "m", "messages": [{"role": "user", "content": "2+2?"}], "temperature": 0.8,
               "max_tokens": 4}
    raw = {"model": "m", "choices": [{"finish_reason": "stop", "message": {"content": "4"}}]}
    evidence = {"schema_version": 1, "request_id": request_id, "request_payload_sha256": G.evidence_digest(payload),
                "response_sha256": G.evidence_digest(raw), "logprob_convention": "sampled_distribution",
                "policy": policy.to_dict(), "finish_reason": "eos", "context_token_ids": [1, 2, 3],
                "action_token_ids": [7, 2], "behavior_log_probs": [-0.1, -0.2], "stop_token_count": 1,
                "context_truncation": "none"}
    return payload, {**raw, "training_evidence": evidence}


def test_valid_evidence_becomes_a_turn():
    policy = _policy()
    contract = G.TrainingGenerationContract(policy, _capabilities(policy))
    payload, completion = _exchange(policy)
    turn = contract.validate(payload, completion, "req-1", 1)
    assert turn.action_token_ids == (7, 2) and turn.behavior_log_probs == (-0.1, -0.2)
    assert turn.finish_reason == "eos" and turn.policy == policy


@pytest.mark.parametrize("tamper", ["request_id", "response", "payload", "policy", "stream", "budget", "evidence",
                                    "finish"])
def test_every_broken_binding_is_rejected(tamper):
    policy = _policy()
    contract = G.TrainingGenerationContract(policy, _capabilities(policy))
    payload, completion = _exchange(policy)
    request_id = "req-1"
    if tamper == "request_id":
        request_id = "req-2"
    elif tamper == "response":
        completion["choices"][0]["message"]["content"] = "5"
    elif tamper == "payload":
        payload["messages"][0]["content"] = "3+3?"
    elif tamper == "policy":
        other = T.PolicyRef(5, policy.digest, "run", dict(policy.identities), dict(policy.sampling))
        completion["training_evidence"]["policy"] = other.to_dict()
    elif tamper == "stream":
        payload["stream"] = True
    elif tamper == "budget":
        payload["max_tokens"] = 1
    elif tamper == "evidence":
        del completion["training_evidence"]
    elif tamper == "finish":
        completion["training_evidence"]["finish_reason"] = "length"
    with pytest.raises(G.TrainingCapabilityError):
        contract.validate(payload, completion, request_id, 1)


def test_capability_receipt_must_cover_the_lease():
    policy = _policy()
    caps = _capabilities(policy)
    with pytest.raises(G.TrainingCapabilityError):
        G.TrainingGenerationContract(policy, {**caps, "full_categorical": False})
    with pytest.raises(G.TrainingCapabilityError):
        G.TrainingGenerationContract(policy, {**caps, "schema_version": 2})
    bare = T.PolicyRef(4, policy.digest, "run")
    with pytest.raises(G.TrainingCapabilityError):
        G.TrainingGenerationContract(bare, _capabilities(bare))


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_digests_and_verdicts_match_the_reference():
    import_reference()
    from rollout_manager import generation_training as R
    from rollout_manager import training as RT

    policy = _policy()
    payload, completion = _exchange(policy)
    assert R.evidence_digest(payload) == G.evidence_digest(payload)
    ref_policy = RT.PolicyRef.from_dict(policy.to_dict())
    ref_turn = R.TrainingGenerationContract(ref_policy, _capabilities(policy)).validate(payload, completion, "req-1", 1)
    ours = G.TrainingGenerationContract(policy, _capabilities(policy)).validate(payload, completion, "req-1", 1)
    assert ours.to_dict() == ref_turn.to_dict()
