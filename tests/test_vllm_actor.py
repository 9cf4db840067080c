"""Owned-engine actor protocol (rollout/vllm_actor.py) with a fake engine on CPU: start, generate,
head updates checked by read-back digest, failure reporting, close."""

import pytest
import torch

from tiny_dsv41_b200.rollout.vllm_actor import GenerationRequest, VLLMActor, tensor_digest

ENGINE = "tests.fake_vllm_engine:FakeEngine"


def test_actor_generate_and_head_update():
    actor = VLLMActor("unused", engine=ENGINE, timeout=120)
    try:
        assert actor.start()["ready"]
        out = actor.generate(GenerationRequest(prompts=[[1, 2, 3], [7]], max_tokens=4))
        assert out[0]["token_ids"] == [4, 5, 6, 7] and out[1]["token_ids"] == [8, 9, 10, 11]
        head = torch.randn(4, 3).bfloat16()
        receipt = actor.update_head(head, version=3)
        assert receipt == {"version": 3, "digest": tensor_digest(head)}
        assert actor.receipt() == receipt
    finally:
        result = actor.close()
    assert result["closed"] and result["version"] == 3


def test_actor_reports_engine_failure():
    actor = VLLMActor("unused", engine=ENGINE, timeout=120, fail_on="generate")
    actor.start()
    with pytest.raises(RuntimeError, match="engine failure"):
        actor.generate(GenerationRequest(prompts=[[1]], max_tokens=1))
    with pytest.raises(RuntimeError):
        actor.receipt()
    actor.close()
