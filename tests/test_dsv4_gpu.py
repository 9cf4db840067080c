"""DeepSeek-V4.1 on the sm_100a kernels (bf16, GPU) vs the fp32 CPU model with the same weights,
plus the mHC kernels against their PyTorch definitions."""

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
from tiny_dsv41_b200.ops import mhc as H

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def test_mhc_kernels_match_reference():
    torch.manual_seed(0)
    comb = torch.randn(37, 4, 4, device="cuda", requires_grad=True)
    out = H.sinkhorn(comb, 20, 1e-6)
    g = torch.randn_like(out)
    out.backward(g)
    cr = comb.detach().clone().requires_grad_()
    ref = H.sinkhorn_reference(cr, 20, 1e-6)
    ref.backward(g)
    assert _rel(out, ref) < 1e-5 and _rel(comb.grad, cr.grad) < 1e-3
    s = torch.randn(37, 4, 264, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.rand(37, 4, device="cuda", requires_grad=True)
    y = H.collapse(s, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    sr, wr = s.detach().float().requires_grad_(), w.detach().clone().requires_grad_()
    H.collapse_reference(sr, wr).backward(gy.float())
    assert _rel(y, H.collapse_reference(sr, wr)) < 1e-2
    assert _rel(s.grad, sr.grad) < 1e-2 and _rel(w.grad, wr.grad) < 1e-2
    v = torch.randn(37, 264, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(37, 4, 264, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    post = torch.rand(37, 4, device="cuda", requires_grad=True)
    cm = torch.rand(37, 4, 4, device="cuda", requires_grad=True)
    e = H.expand(v, r, post, cm)
    ge = torch.randn_like(e)
    e.backward(ge)
    vr, rr = v.detach().float().requires_grad_(), r.detach().float().requires_grad_()
    pr, cr2 = post.detach().clone().requires_grad_(), cm.detach().clone().requires_grad_()
    er = H.expand_reference(vr, rr, pr, cr2)
    er.backward(ge.float())
    assert _rel(e, er) < 1e-2
    for a, b in ((v, vr), (r, rr), (post, pr), (cm, cr2)):
        assert _rel(a.grad, b.grad) < 1e-2
    ops.check_status("mhc")


def test_hyper_connection_module_gpu_vs_cpu():
    from tiny_dsv41_b200.models.dsv4.mhc import HyperConnection

    torch.manual_seed(3)
    cfg = DeepSeekV41Config.tiny()
    ref = HyperConnection(cfg)
    torch.nn.init.normal_(ref.fn, std=0.02)
    torch.nn.init.normal_(ref.base, std=0.1)
    gpu = HyperConnection(cfg).cuda()
    gpu.load_state_dict(ref.state_dict())
    streams = torch.randn(2, 16, 4, cfg.hidden_size).to(torch.bfloat16)
    pre_in = torch.rand(2, 16, 4)
    outs_g = gpu(streams.cuda(), pre_in.cuda())
    outs_r = ref(streams.float(), pre_in)
    grads = [torch.randn_like(o.float()) for o in outs_r[1:]]
    torch.autograd.backward([o.float() for o in outs_g[1:]], [g.cuda() for g in grads])
    torch.autograd.backward([o.float() for o in outs_r[1:]], grads)
    for name in ("fn", "base", "scale"):
        err = _rel(getattr(gpu, name).grad, getattr(ref, name).grad)
        assert err < 2e-2, (name, err)


def test_dsv4_tiny_gpu_matches_cpu():
    torch.manual_seed(0)
    cfg = DeepSeekV41Config.tiny()
    ref = DeepSeekV41ForCausalLM(cfg)
    islands = {id(p) for p in ref.fp32_island_parameters()}
    with torch.no_grad():  # both sides start from the same bf16-representable weights
        for p in ref.parameters():
            if id(p) not in islands:
                p.copy_(p.to(torch.bfloat16).float())
    gpu = DeepSeekV41ForCausalLM(cfg)
    gpu.load_state_dict(ref.state_dict())
    gpu = gpu.cuda().to_mixed_precision(torch.bfloat16)
    ids = torch.randint(0, 32, (2, 64))
    a = gpu(ids.cuda(), labels=ids.cuda())
    b = ref(ids, labels=ids)
    assert abs(a.loss.item() - b.loss.item()) / b.loss.item() < 3e-2
    a.loss.backward()
    b.loss.backward()
    ref_params = dict(ref.named_parameters())
    bad = []
    for name, p in gpu.named_parameters():
        q = ref_params[name]
        if q.grad is None or q.grad.norm() == 0:
            continue
        if name.endswith("hc.base") or name.endswith("hc.scale"):
            continue  # token sums of nearly cancelling terms; covered by the module-level test above
        # direction check: sums over tokens (mHC base, norms) cancel strongly, so bf16 vs fp32
        # magnitudes can differ more than the gradient direction does
        cos = torch.nn.functional.cosine_similarity(p.grad.float().cpu().flatten(), q.grad.float().flatten(), dim=0)
        if cos < 0.9:
            bad.append((name, cos.item()))
    assert not bad, bad
    ops.check_status("dsv4 tiny")
