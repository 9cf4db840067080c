"""Cache fake quantization (FP8 / FP4 KV-cache emulation for DeepSeek-V4 scoring)."""

import pytest
import torch

from tiny_dsv41_b200.ops import quant as Q


def test_e2m1_grid_and_ties():
    v = torch.tensor([0.0, 0.25, 0.26, 0.74, 0.75, 1.25, 1.3, 1.75, 2.5, 2.6, 3.5, 5.0, 5.1, 6.0, -0.75, -0.2])
    want = [0.0, 0.0, 0.5, 0.5, 1.0, 1.0, 1.5, 2.0, 2.0, 3.0, 4.0, 4.0, 6.0, 6.0, -1.0, -0.0]
    got = Q._e2m1_round(v)
    assert got.tolist() == want
    assert torch.signbit(got[-1])


def test_block_scales():
    x = torch.zeros(1, 32)
    x[0, 0] = 3.0  # amax 3 -> fp4_index scale 2^ceil(log2(0.5)) = 0.5; fp8 scale 2^ceil(log2(3/448)) = 2^-7
    x[0, 1] = 0.3
    y = Q.fake_quant_reference(x, "fp4_index")
    assert y[0, 0].item() == 3.0 and y[0, 1].item() == 0.25  # 0.3 / 0.5 = 0.6 -> 0.5 -> 0.25
    y8 = Q.fake_quant_reference(x, "fp8")
    assert y8[0, 0].item() == 3.0 and abs(y8[0, 1].item() - 0.3) < 0.3 * 2 ** -3
    xk = torch.zeros(1, 16)
    xk[0, 0] = 6.0  # fp4_kv scale = e4m3(1.0) = 1
    xk[0, 1] = 2.6
    yk = Q.fake_quant_reference(xk, "fp4_kv")
    assert yk[0, 0].item() == 6.0 and yk[0, 1].item() == 3.0


def test_unaligned_width_passes_through_and_gradient_is_identity():
    x = torch.randn(2, 10, requires_grad=True)
    assert Q.quantize_activation(x, "fp8") is not None
    assert torch.equal(Q.fake_quant_reference(x.detach(), "fp4_kv"), x.detach())
    y = torch.randn(3, 64, requires_grad=True)
    out = Q.quantize_activation(y, "fp4_kv")
    assert not torch.equal(out.detach(), y.detach())
    out.sum().backward()
    assert torch.equal(y.grad, torch.ones_like(y))


def test_dsv4_hf_cache_quantization_runs_and_changes_scores():
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM

    torch.manual_seed(0)
    cfg = DeepSeekV41Config.tiny()
    ids = torch.randint(3, cfg.vocab_size, (1, 24))
    losses = []
    for mode in ("none", "hf"):
        torch.manual_seed(0)
        model = DeepSeekV41ForCausalLM(DeepSeekV41Config.from_dict({**cfg.to_dict(), "cache_quantization": mode}))
        out = model(ids, labels=ids)
        out.loss.backward()
        assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())
        losses.append(out.loss.item())
    assert losses[0] != losses[1] and abs(losses[0] - losses[1]) < 0.5
    with pytest.raises(ValueError):
        DeepSeekV41Config.from_dict({**cfg.to_dict(), "cache_quantization": "int8"})


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["fp8", "fp4_index", "fp4_kv"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_cuda_kernel_matches_reference(kind, dtype):
    from tiny_dsv41_b200 import ops

    torch.manual_seed(1)
    x = (torch.randn(7, 3, 512) * torch.logspace(-3, 2, 512)).to(dtype)
    want = Q.fake_quant_reference(x, kind)
    got = ops.ext().cache_fake_quant(x.cuda(), Q.KINDS[kind][0]).cpu()
    assert torch.equal(got, want)
