"""HF Qwen3-MoE safetensors loader/writer: round trip, EP slicing, and the reference loader's view."""

import pytest
import torch

from tests.ref_oracle import import_reference, reference_available
from tiny_dsv41_b200.models.qwen import (Qwen3MoeConfig, Qwen3MoeForCausalLM, hf_tensor_names, load_qwen3_moe,
                                         save_qwen3_moe)


def _cfg():
    return Qwen3MoeConfig.tiny(num_hidden_layers=2, max_window_layers=2)


def test_roundtrip(tmp_path):
    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(_cfg())
    save_qwen3_moe(model, tmp_path, shard_size=1 << 20)
    loaded = load_qwen3_moe(tmp_path, dtype=None)
    for (k, a), b in zip(model.state_dict().items(), loaded.state_dict().values()):
        assert torch.equal(a, b), k
    import json

    names = json.loads((tmp_path / "model.safetensors.index.json").read_text())["weight_map"]
    assert sorted(names) == sorted(hf_tensor_names(_cfg()))


def test_expert_slice(tmp_path):
    torch.manual_seed(1)
    model = Qwen3MoeForCausalLM(_cfg())
    save_qwen3_moe(model, tmp_path)

    class Half:  # an EP rank that owns experts [4, 8)
        def expert_range(self, n):
            return n // 2, n

        def __getattr__(self, name):
            from tiny_dsv41_b200.parallel.dispatch import TokenDispatcher

            return getattr(TokenDispatcher(), name)

    part = load_qwen3_moe(tmp_path, dtype=None, token_dispatcher=Half())
    full = model.model.layers[1].mlp.experts.gate_up_proj
    assert torch.equal(part.model.layers[1].mlp.experts.gate_up_proj, full[4:])


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_reference_loader_reads_our_files(tmp_path):
    import_reference()
    from dsv41_train.models.qwen.checkpoint import load_qwen3_moe as ref_load

    torch.manual_seed(2)
    model = Qwen3MoeForCausalLM(_cfg())
    save_qwen3_moe(model, tmp_path)
    ref = ref_load(tmp_path, dtype=None)
    ours = model.state_dict()
    for name, value in ref.state_dict().items():
        assert torch.equal(value, ours[name]), name
