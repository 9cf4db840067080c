"""LoRA injection, adapter file round trips, merge/unmerge, and loading adapters the reference wrote."""

import pytest
import torch

from tiny_dsv41_b200.lora import (LoRAConfig, LoRALinear, adapter_parameters, inject_lora, load_adapter,
                                  merge_adapters, read_adapter, save_adapter, unmerge_adapters)
from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM

from ref_oracle import import_reference, reference_available


def _model():
    torch.manual_seed(0)
    return DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny())


def test_inject_train_save_load_roundtrip(tmp_path):
    model = _model()
    names = inject_lora(model, LoRAConfig(rank=4, alpha=8.0, targets=("attention.q_a",)))
    assert len(names) == 6
    trainable = [p for p in model.parameters() if p.requires_grad]
    assert len(trainable) == 12 and all(any(p is q for q in adapter_parameters(model)) for p in trainable)
    ids = torch.randint(0, 32, (1, 20))
    model(ids, labels=ids).loss.backward()
    assert all(p.grad is not None for p in adapter_parameters(model))
    with torch.no_grad():
        for p in adapter_parameters(model):
            p.add_(0.01)
    path = tmp_path / "adapter.pt"
    save_adapter(model, path, base_identity={"config_sha256": "x"})
    other = _model()
    inject_lora(other, LoRAConfig(rank=4, alpha=8.0, targets=("attention.q_a",)))
    load_adapter(other, path, base_identity={"config_sha256": "x"})
    with pytest.raises(ValueError):
        load_adapter(other, path, base_identity={"config_sha256": "y"})
    model.eval(), other.eval()
    with torch.no_grad():
        a = model(ids).logits
        b = other(ids).logits
        assert torch.allclose(a, b, atol=1e-6)
        merge_adapters(other)
        c = other(ids).logits
        assert torch.allclose(a, c, atol=1e-4)
        state = other.state_dict()
        unmerge_adapters(other)
    assert torch.equal(state["model.layers.0.attention.q_a.weight"], model.model.layers[0].attention.q_a.weight)


@pytest.mark.skipif(not reference_available(), reason="reference not installed under baseline/_ref")
def test_reads_reference_adapter(tmp_path):
    import_reference()
    from dsv41_train.lora import LoRAConfig as RefConfig
    from dsv41_train.lora import inject_lora as ref_inject
    from dsv41_train.lora import save_adapter as ref_save
    from dsv41_train.models.dsv4.config import DeepSeekV41Config as RefCfg
    from dsv41_train.models.dsv4.model import DeepSeekV41ForCausalLM as RefModel

    torch.manual_seed(1)
    ref = RefModel(RefCfg.tiny())
    ref_inject(ref, RefConfig(rank=4, alpha=8.0, targets=("attention.q_a", "attention.o_b")))
    path = tmp_path / "ref_adapter.pt"
    ref_save(ref, path, base_identity={"k": 1})
    mine = _model()
    inject_lora(mine, LoRAConfig(rank=4, alpha=8.0, targets=("attention.q_a", "attention.o_b")))
    load_adapter(mine, path, base_identity={"k": 1})
    payload = read_adapter(path)
    for name, value in payload["weights"].items():
        assert torch.equal(mine.get_parameter(name), value)
