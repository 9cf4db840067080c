"""Training evidence from an existing generation (chat-completion) route, checked fail-closed.

A serving route can feed GRPO only if it returns, for each request, the exact tokens it sampled,
their behavior log-probabilities under the sampled (full categorical) distribution, and a receipt
of the policy it had loaded, all bound by digest to the dispatched request and the raw response.
Nothing here reconstructs tokens or probabilities from text: a response without that evidence is
rejected. Same contract and digests as ``rollout_manager/generation_training.py`` of the reference
(the receipt and evidence formats are what a serving implementation emits, so they must agree).

    contract = TrainingGenerationContract(policy_ref, capability_receipt)
    contract.check_payload(request)                     # before the request leaves the process
    turn = contract.validate(request, completion, request_id, turn_id)   # -> TurnTrace
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Mapping

from .training import PolicyRef, TurnTrace

_CAPABILITIES = ("token_ids", "sampled_token_logprobs", "loaded_policy_identity", "request_response_binding",
                 "full_categorical")
_HEX = frozenset("0123456789abcdef")


class TrainingCapabilityError(ValueError):
    """The route cannot supply (or did not supply) the evidence a training turn needs."""


def evidence_digest(value) -> str:
    """sha256 of the canonical JSON form: sorted keys, no spaces, ASCII, no NaN / inf."""
    text = json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=True, allow_nan=False)
    return hashlib.sha256(text.encode()).hexdigest()


def _is_sha256(value) -> bool:
    return isinstance(value, str) and len(value) == 64 and set(value) <= _HEX


def _schema_v1(value) -> bool:
    return isinstance(value, Mapping) and type(value.get("schema_version")) is int and value["schema_version"] == 1


class TrainingGenerationContract:
    REQUIRED = _CAPABILITIES

    def __init__(self, policy, capabilities) -> None:
        if isinstance(policy, Mapping):
            policy = PolicyRef.from_dict(policy)
        if not isinstance(policy, PolicyRef):
            raise TrainingCapabilityError("a training route needs the leased PolicyRef")
        if not _schema_v1(capabilities):
            raise TrainingCapabilityError("a training route needs a serving capability receipt of schema_version 1")
        missing = [name for name in _CAPABILITIES if capabilities.get(name) is not True]
        if missing:
            raise TrainingCapabilityError("the serving route does not declare: " + ", ".join(missing))
        if capabilities.get("logprob_convention") != "sampled_distribution":
            raise TrainingCapabilityError("behavior log-probabilities must be those of the sampled distribution")
        if capabilities.get("policy") != policy.to_dict():
            raise TrainingCapabilityError("the capability receipt names a different policy than the lease")
        for name in ("tokenizer_sha256", "chat_template_sha256"):
            if not _is_sha256(policy.identities.get(name)):
                raise TrainingCapabilityError(f"the leased policy needs an exact {name}")
        self.policy = policy
        self.capabilities = dict(capabilities)

    def check_payload(self, payload) -> None:
        """Reject, before dispatch, a request whose sampling or shape cannot yield a training turn."""
        if not isinstance(payload, dict):
            raise TrainingCapabilityError("a generation request must be a mapping")
        want = self.policy.sampling
        if (payload.get("temperature") != want["temperature"] or payload.get("top_p", 1) != want["top_p"]
                or payload.get("top_k", 0) != want["top_k"]):
            raise TrainingCapabilityError("request sampling differs from the leased full categorical policy")
        if payload.get("stream", False) is not False or payload.get("n", 1) != 1:
            raise TrainingCapabilityError("a training request is one complete, non-streaming choice")
        budget = payload.get("max_tokens")
        if type(budget) is not int or budget < 1:
            raise TrainingCapabilityError("a training request needs an explicit positive max_tokens")
        evidence_digest(payload)  # canonical JSON must exist before the request is observable

    def validate(self, payload, completion, request_id: str, turn_id: int) -> TurnTrace:
        self.check_payload(payload)
        if not isinstance(completion, dict):
            raise TrainingCapabilityError("the completion must be the raw serving response")
        evidence = completion.get("training_evidence")
        if not _schema_v1(evidence):
            raise TrainingCapabilityError("the response carries no training_evidence of schema_version 1")
        if evidence.get("request_id") != request_id:
            raise TrainingCapabilityError("the evidence belongs to another request")
        if evidence.get("request_payload_sha256") != evidence_digest(payload):
            raise TrainingCapabilityError("the evidence is not bound to the dispatched request")
        raw = {key: value for key, value in completion.items() if key != "training_evidence"}
        if evidence.get("response_sha256") != evidence_digest(raw):
            raise TrainingCapabilityError("the evidence is not bound to the raw response")
        if evidence.get("logprob_convention") != "sampled_distribution":
            raise TrainingCapabilityError("the evidence uses another log-probability convention")
        try:
            loaded = PolicyRef.from_dict(evidence.get("policy", {}))
        except (TypeError, ValueError) as error:
            raise TrainingCapabilityError("the evidence carries no valid policy receipt") from error
        if loaded != self.policy:
            raise TrainingCapabilityError("the loaded policy differs from the group's lease")
        if not isinstance(payload.get("model"), str) or completion.get("model") != payload["model"]:
            raise TrainingCapabilityError("the response names another model than the request")
        choices = completion.get("choices")
        if not isinstance(choices, list) or len(choices) != 1 or not isinstance(choices[0], dict):
            raise TrainingCapabilityError("the response must hold exactly one raw choice")
        finish = evidence.get("finish_reason")
        if choices[0].get("finish_reason") != ("stop" if finish == "eos" else finish):
            raise TrainingCapabilityError("the evidence finish reason disagrees with the raw choice")
        actions = evidence.get("action_token_ids")
        if not isinstance(actions, list) or len(actions) > payload["max_tokens"]:
            raise TrainingCapabilityError("the sampled tokens exceed the request's token budget")
        try:
            return TurnTrace(turn_id=turn_id, request_id=request_id, context_token_ids=evidence["context_token_ids"],
                             action_token_ids=actions, behavior_log_probs=evidence["behavior_log_probs"],
                             policy=loaded, finish_reason=finish, stop_token_count=evidence["stop_token_count"],
                             context_truncation=evidence["context_truncation"])
        except (KeyError, TypeError, ValueError) as error:
            raise TrainingCapabilityError("invalid token / log-probability evidence") from error


__all__ = ["TrainingCapabilityError", "TrainingGenerationContract", "evidence_digest"]
