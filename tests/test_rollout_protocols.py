"""Training records and LoRA update packets: round trips, rejection rules and byte-level
compatibility with the reference implementations (records and packets cross in both directions)."""

import hashlib
import socket

import pytest
import torch

from tests.ref_oracle import import_reference, reference_available
from tiny_dsv41_b200.rollout import training as T
from tiny_dsv41_b200.rollout.lora_transport import (pack_update, receive_update, send_update, unpack_update,
                                                    validate_update)

DIGEST = hashlib.sha256(b"policy").hexdigest()
RESET = hashlib.sha256(b"reset").hexdigest()


def _group(rewards=(1.0, 0.0)):
    policy = T.PolicyRef(3, DIGEST, "run-a", {"engine": "native"})
    prompt = [1, 2, 3]
    samples = [T.TrainingTrajectory(7, "task/0", T.token_digest(prompt), RESET, i,
                                    (T.TurnTrace(1, f"r{i}", prompt, [4, 5], [-0.5, -1.0], policy, "eos", 1),), r)
               for i, r in enumerate(rewards)]
    return T.TrainingGroup(7, "task/0", T.token_digest(prompt), RESET, policy, len(samples), samples)


def test_records_roundtrip_and_rules():
    group = _group()
    text = T.dumps(group)
    assert T.loads(text) == group
    assert T.to_rollout_group(group).samples[0].response_ids == [4, 5]
    with pytest.raises(ValueError):
        T.loads(text.replace('"schema_version":1', '"schema_version":2'))
    with pytest.raises(ValueError):  # missing reward is not zero
        _group(rewards=(1.0, None))
    with pytest.raises(ValueError):
        T.PolicyRef(1, DIGEST, "x", sampling={"temperature": 1.0, "top_p": 0.9, "top_k": 0})


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_records_match_reference_format():
    import_reference()
    from rollout_manager import training as R

    text = T.dumps(_group())
    ref = R.loads(text)
    assert R.dumps(ref) == text
    assert T.dumps(T.loads(R.dumps(ref))) == text
    assert R.token_digest([1, 2, 3]) == T.token_digest([1, 2, 3])


def _tensors():
    g = torch.Generator().manual_seed(0)
    return {"language_model.model.layers.0.attn.wq_a.lora_A.weight": torch.randn(8, 16, generator=g).bfloat16(),
            "language_model.model.layers.0.attn.wq_a.lora_B.weight": torch.randn(32, 8, generator=g).bfloat16()}


def test_lora_packet_roundtrip_and_tamper():
    manifest, payload = pack_update(_tensors(), version=2, lineage="run", adapter_id=1,
                                    peft={"r": 8, "lora_alpha": 8.0, "target_modules": ["wq_a"]},
                                    base_identity={"config_sha256": DIGEST, "index_sha256": DIGEST})
    out = unpack_update(manifest, payload)
    for name, t in _tensors().items():
        assert torch.equal(out[name], t)
    bad = bytearray(payload)
    bad[0] ^= 1
    with pytest.raises(ValueError):
        validate_update(manifest, bytes(bad))
    a, b = socket.socketpair()
    try:
        send_update(a, manifest, payload)
        got = receive_update(b)
    finally:
        a.close()
        b.close()
    assert got == (manifest, payload)


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_lora_packet_matches_reference():
    import_reference()
    from rollout_manager.backends import vllm_lora_transport as R

    args = dict(version=2, lineage="run", adapter_id=1, peft={"r": 8, "lora_alpha": 8.0, "target_modules": ["wq_a"]},
                base_identity={"config_sha256": DIGEST, "index_sha256": DIGEST})
    ours = pack_update(_tensors(), **args)
    theirs = R.pack_update(_tensors(), **args)
    assert ours == theirs
    R.validate_update(*ours)


def test_export_q_a_update_from_dsv4_learner():
    from tiny_dsv41_b200.lora import inject_lora
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
    from tiny_dsv41_b200.rl.lora_config import DistributedLoRAConfig
    from tiny_dsv41_b200.rl.lora_export import export_q_a_update

    torch.manual_seed(0)
    model = DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()).to(torch.bfloat16)
    profile = DistributedLoRAConfig(rank=8, alpha=16.0, layers=(0, 2))
    for p in model.parameters():
        p.requires_grad_(False)
    for layer in (0, 2):
        inject_lora(model.model.layers[layer], profile.lora_config())
    manifest, payload = export_q_a_update(model, version=0, lineage="run", adapter_id=1, lora_config=profile,
                                          base_identity={"config_sha256": DIGEST, "index_sha256": DIGEST})
    names = [t["name"] for t in manifest["tensors"]]
    assert names == sorted(f"language_model.model.layers.{i}.attn.wq_a.lora_{x}.weight" for i in (0, 2) for x in "AB")
    assert manifest["peft"] == {"r": 8, "lora_alpha": 16.0, "target_modules": ["wq_a"]}
    validate_update(manifest, payload)
