"""Qwen3-MoE on the sm_100a kernels (bf16, GPU) against the fp32 CPU model with the same weights."""

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def test_qwen_tiny_gpu_matches_cpu():
    torch.manual_seed(0)
    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=512, hidden_size=256, num_experts=8,
                              num_experts_per_tok=2, moe_intermediate_size=128)
    ref = Qwen3MoeForCausalLM(cfg)
    with torch.no_grad():  # well-separated router logits: bf16 and fp32 pick the same experts
        for layer in ref.model.layers:
            layer.mlp.gate.weight.mul_(10.0)
    with torch.no_grad():  # both sides start from the same bf16-representable weights
        for p in ref.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    gpu = Qwen3MoeForCausalLM(cfg)
    gpu.load_state_dict(ref.state_dict())
    gpu = gpu.cuda().to(torch.bfloat16)
    ids = torch.randint(0, 512, (2, 128))
    labels = ids.clone()
    labels[:, :64] = -100
    a = gpu(ids.cuda(), labels=labels.cuda(), output_router_logits=True)
    b = ref(ids, labels=labels, output_router_logits=True)
    assert abs(a.loss.item() - b.loss.item()) / b.loss.item() < 2e-2
    a.loss.backward()
    b.loss.backward()
    ref_params = dict(ref.named_parameters())
    for name, p in gpu.named_parameters():
        q = ref_params[name]
        assert p.grad is not None, name
        err = _rel(p.grad, q.grad)
        # the router gradient goes through softmax differences of bf16 logits
        # the router (and, through it, the embedding) gradient goes through softmax differences of
        # bf16 logits; everything else is a plain bf16-vs-fp32 comparison
        tol = 0.15 if name.endswith("mlp.gate.weight") else 0.1
        assert err < tol, (name, err)
    ops.check_status("qwen tiny")


def test_qwen_training_step_reduces_loss():
    from tiny_dsv41_b200.optim import FusedAdamW

    torch.manual_seed(1)
    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=512)
    model = Qwen3MoeForCausalLM(cfg).cuda().to(torch.bfloat16)
    model.gradient_checkpointing_enable()
    opt = FusedAdamW(model.parameters(), lr=3e-3, in_backward=True)
    ids = torch.randint(0, 512, (1, 256), device="cuda")
    losses = []
    for _ in range(8):
        opt.begin_step()
        out = model(ids, labels=ids, output_router_logits=True)
        out.loss.backward()
        losses.append(out.loss.item())
    assert losses[-1] < losses[0] - 0.5, losses


def test_kv_cache_decoding_gpu():
    from tiny_dsv41_b200.models.qwen.generation import IncrementalLogits

    torch.manual_seed(4)
    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=512)
    model = Qwen3MoeForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    inc = IncrementalLogits(model)
    ids = [1, 17, 33, 250, 9, 77, 3]
    with torch.no_grad():
        for _ in range(5):
            seq = torch.tensor([ids], device="cuda")
            a = inc(seq).float()
            b = model(seq).logits[:, -1].float()
            assert _rel(a, b) < 2e-2
            ids.append(int(b.argmax()))
    assert inc.prefills == 1


def test_checkpoint_recompute_reuses_attention_and_matches_plain_backward():
    """With gradient checkpointing the recompute reuses the first pass's attention output
    (parallel/replay.py); the gradients must equal those of the same model without checkpointing."""
    torch.manual_seed(3)
    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=512)
    plain = Qwen3MoeForCausalLM(cfg).cuda().to(torch.bfloat16)
    ckpt = Qwen3MoeForCausalLM(cfg).cuda().to(torch.bfloat16)
    ckpt.load_state_dict(plain.state_dict())
    ckpt.gradient_checkpointing_enable()
    ids = torch.randint(0, 512, (1, 256), device="cuda")
    calls = {"n": 0}
    a = plain(ids, labels=ids, output_router_logits=True)
    a.loss.backward()
    from tiny_dsv41_b200.ops import _ext

    module = _ext._ext
    original = module.attn_fwd

    def counting(*args):
        calls["n"] += 1
        return original(*args)

    try:
        _ext._ext = type("Wrapped", (), {"__getattr__": lambda self, n: counting if n == "attn_fwd"
                                         else getattr(module, n)})()
        b = ckpt(ids, labels=ids, output_router_logits=True)
        b.loss.backward()
    finally:
        _ext._ext = module
    assert calls["n"] == cfg.num_hidden_layers  # forward only: the recompute ran no attention kernel
    assert abs(a.loss.item() - b.loss.item()) < 1e-3
    grads = dict(plain.named_parameters())
    for name, p in ckpt.named_parameters():
        err = _rel(p.grad, grads[name].grad)
        assert err < 2e-2, (name, err)
