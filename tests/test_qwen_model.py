"""Qwen3-MoE: CPU parity of loss and gradients against the reference implementation."""

import pytest
import torch

from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM

from ref_oracle import import_reference, reference_available


def _tiny():
    return Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=64, num_experts=8, num_experts_per_tok=2)


def test_config_roundtrip(tmp_path):
    cfg = _tiny()
    path = tmp_path / "config.json"
    import json

    path.write_text(json.dumps(cfg.to_dict()))
    assert Qwen3MoeConfig.from_json(path) == cfg
    with pytest.raises(ValueError):
        Qwen3MoeConfig.tiny(num_key_value_heads=3)


def test_forward_backward_cpu():
    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(_tiny())
    ids = torch.randint(0, 64, (2, 16))
    out = model(ids, labels=ids, output_router_logits=True)
    assert torch.isfinite(out.loss)
    out.loss.backward()
    assert model.model.layers[0].mlp.experts.gate_up_proj.grad is not None


@pytest.mark.skipif(not reference_available(), reason="reference not installed under baseline/_ref")
def test_parity_with_reference_cpu():
    import_reference()
    from dsv41_train.models.qwen.config import Qwen3MoeConfig as RefConfig
    from dsv41_train.models.qwen.model import Qwen3MoeForCausalLM as RefModel

    torch.manual_seed(0)
    cfg = _tiny()
    mine = Qwen3MoeForCausalLM(cfg)
    ref = RefModel(RefConfig(**cfg.to_dict()))
    missing, unexpected = ref.load_state_dict(mine.state_dict(), strict=False)
    assert not unexpected and not missing
    ids = torch.randint(0, 64, (2, 24))
    labels = ids.clone()
    labels[:, :12] = -100
    a = mine(ids, labels=labels, output_router_logits=True)
    b = ref(ids, labels=labels, output_router_logits=True)
    assert torch.allclose(a.loss, b.loss, rtol=1e-5, atol=1e-6), (a.loss, b.loss)
    assert torch.allclose(a.aux_loss, b.aux_loss, rtol=1e-5)
    a.loss.backward()
    b.loss.backward()
    ref_params = dict(ref.named_parameters())
    for name, p in mine.named_parameters():
        q = ref_params[name]
        assert p.grad is not None and q.grad is not None, name
        err = (p.grad - q.grad).norm() / q.grad.norm().clamp_min(1e-12)
        assert err < 1e-4, (name, err.item())


def test_kv_cache_sampling_matches_full_forward():
    from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig as Cfg
    from tiny_dsv41_b200.rl.data import PromptRecord
    from tiny_dsv41_b200.rl.policy import QwenPolicy
    from tiny_dsv41_b200.rl.rollout import generate_group

    torch.manual_seed(0)
    cfg = Cfg.tiny(num_hidden_layers=2, max_window_layers=2, vocab_size=64)
    from tiny_dsv41_b200.models.qwen import Qwen3MoeForCausalLM as M

    policy = QwenPolicy(M(cfg), trainable_scope="lm_head")
    record = PromptRecord([1, 5, 7, 9], target_ids=[3, 3])
    runs = []
    for cached in (False, True):
        policy.qwen_kv_cache = cached
        policy._session = None
        gen = torch.Generator().manual_seed(3)
        runs.append(generate_group(policy, record, 2, 6, 1.0, eos_token_id=None, policy_version=0, group_id=0,
                                   generator=gen))
    for a, b in zip(runs[0].samples, runs[1].samples):
        assert a.response_ids == b.response_ids
        assert a.behavior_log_probs == pytest.approx(b.behavior_log_probs, abs=1e-5)
    assert policy._session.prefills == 2  # one per sample, every later token is incremental


def test_flash_attention_eligibility():
    """The tcgen05 attention takes only the plain causal case it implements; everything else
    (masks, dropout, other head dims, ragged lengths) stays on scaled-dot-product attention."""
    from tiny_dsv41_b200.ops import attention as A

    def t(b, l, h, d, dtype=torch.bfloat16):
        return torch.zeros(b, l, h, d, dtype=dtype)

    assert A.flash_supported(t(1, 256, 8, 128), t(1, 256, 2, 128), t(1, 256, 2, 128))
    assert not A.flash_supported(t(1, 200, 8, 128), t(1, 200, 2, 128), t(1, 200, 2, 128))  # L % 128
    assert not A.flash_supported(t(1, 256, 8, 64), t(1, 256, 2, 64), t(1, 256, 2, 64))  # head dim
    assert not A.flash_supported(t(1, 256, 6, 128), t(1, 256, 4, 128), t(1, 256, 4, 128))  # GQA groups
    assert not A.flash_supported(*(t(1, 256, 4, 128, torch.float32) for _ in range(3)))  # dtype
    q = torch.randn(1, 256, 4, 128)
    out = A.causal_attention(q, q[:, :, :2], q[:, :, :2])  # CPU: the SDPA path
    assert out.shape == q.shape and torch.isfinite(out).all()
