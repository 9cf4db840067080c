"""DeepSeek-V4.1: CPU parity of loss, gradients and selected-token log-probs with the reference."""

import pytest
import torch

from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM

from ref_oracle import import_reference, reference_available


def test_tiny_config_and_validation():
    cfg = DeepSeekV41Config.tiny()
    assert cfg.num_hidden_layers == 6 and cfg.compress_ratios == [0, 2, 2, 1, 1, 1]
    values = cfg.to_dict()
    values["compress_ratios"] = values["compress_ratios"] + [0, 0]
    values["num_nextn_predict_layers"] = 2
    assert DeepSeekV41Config.from_dict({"text_config": values}).compress_ratios == cfg.compress_ratios
    bad = cfg.to_dict()
    bad["scoring_func"] = "relu"
    with pytest.raises(ValueError):
        DeepSeekV41Config.from_dict(bad)


def test_forward_backward_cpu():
    torch.manual_seed(0)
    model = DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny())
    ids = torch.randint(0, 32, (2, 40))
    out = model(ids, labels=ids)
    assert torch.isfinite(out.loss)
    out.loss.backward()
    assert model.model.layers[1].moe.routed.gate_up.grad is not None
    assert model.model.layers[3].attention.sinks.weight.grad is not None


@pytest.mark.skipif(not reference_available(), reason="reference not installed under baseline/_ref")
def test_parity_with_reference_cpu():
    import_reference()
    from dsv41_train.models.dsv4.config import DeepSeekV41Config as RefConfig
    from dsv41_train.models.dsv4.model import DeepSeekV41ForCausalLM as RefModel

    torch.manual_seed(0)
    cfg = DeepSeekV41Config.tiny()
    mine = DeepSeekV41ForCausalLM(cfg)
    ref = RefModel(RefConfig.tiny())
    missing, unexpected = ref.load_state_dict(mine.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    ids = torch.randint(0, 32, (2, 48))
    mask = torch.ones_like(ids, dtype=torch.bool)
    mask[1, -5:] = False
    seq = torch.zeros_like(ids)
    seq[0, 20:] = 1
    a = mine(ids, attention_mask=mask, labels=ids, sequence_ids=seq)
    b = ref(ids, attention_mask=mask, labels=ids, sequence_ids=seq)
    assert torch.allclose(a.loss, b.loss, rtol=1e-5, atol=1e-6), (a.loss, b.loss)
    a.loss.backward()
    b.loss.backward()
    ref_params = dict(ref.named_parameters())
    for name, p in mine.named_parameters():
        q = ref_params[name]
        if q.grad is None:
            assert p.grad is None or p.grad.abs().max() == 0, name
            continue
        assert p.grad is not None, name
        err = (p.grad - q.grad).norm() / q.grad.norm().clamp_min(1e-12)
        assert err < 1e-4, (name, err.item())
    with torch.no_grad():
        tgt = torch.roll(ids, -1, dims=1)
        la = mine(ids, target_ids=tgt, temperature=0.7).token_log_probs
        lb = ref(ids, target_ids=tgt, temperature=0.7).token_log_probs
    assert torch.allclose(la, lb, atol=1e-5)
