"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import pytest
import torch
import torch.nn.functional as F

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.ops import gemm as G
from tiny_dsv41_b200.ops import moe as M
from tiny_dsv41_b200.ops import norm as N
from tiny_dsv41_b200.ops import rope as R
from tiny_dsv41_b200.ops import router as RT

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    ops.check_status("test")


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (200, 136, 72), (1000, 384, 320), (128, 128, 64)])
def test_gemm_dense(a_mn, b_mn, m, n, k):
    torch.manual_seed(0)
    a = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=DEV, dtype=torch.bfloat16)
    ref = a.float() @ b.float().t()
    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    out = torch.empty(m, n, device=DEV, dtype=torch.float32)
    ops.ext().gemm(a_in, b_in, out, a_mn, b_mn, False)
    assert _rel(out, ref) < 1e-5
    out_bf = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    ops.ext().gemm(a_in, b_in, out_bf, a_mn, b_mn, False)
    assert _rel(out_bf, ref) < 5e-3
    acc = torch.ones(m, n, device=DEV, dtype=torch.float32)
    ops.ext().gemm(a_in, b_in, acc, a_mn, b_mn, True)
    assert _rel(acc, ref + 1) < 1e-5


def test_gemm_large_k():
    torch.manual_seed(1)
    a = torch.randn(512, 4096, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(1024, 4096, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(512, 1024, device=DEV, dtype=torch.float32)
    ops.ext().gemm(a, b, out, False, False, False)
    assert _rel(out, a.float() @ b.float().t()) < 1e-5


def _segments(sizes, block=128):
    padded = [((s + block - 1) // block) * block for s in sizes]
    offs = [0]
    for p in padded[:-1]:
        offs.append(offs[-1] + p)
    return padded, offs


@pytest.mark.parametrize("b_mn", [False, True])
def test_grouped_gemm_m(b_mn):
    torch.manual_seed(2)
    sizes = [100, 0, 300, 128, 5]
    padded, offs = _segments(sizes)
    rows = sum(padded)
    k, n = 192, 384
    x = torch.zeros(rows, k, device=DEV, dtype=torch.bfloat16)
    for s, o in zip(sizes, offs):
        x[o:o + s] = torch.randn(s, k, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(len(sizes), n, k, device=DEV, dtype=torch.bfloat16)
    w_in = w.transpose(1, 2).contiguous() if b_mn else w
    out = torch.full((rows, n), float("nan"), device=DEV, dtype=torch.bfloat16)
    ops.ext().grouped_gemm_m(x, w_in, torch.tensor(offs, dtype=torch.int32, device=DEV),
                             torch.tensor(padded, dtype=torch.int32, device=DEV), out, b_mn, rows)
    for g, (s, o, p) in enumerate(zip(sizes, offs, padded)):
        if p == 0:
            continue
        ref = x[o:o + p].float() @ w[g].float().t()
        assert _rel(out[o:o + p], ref) < 5e-3


def test_grouped_gemm_k():
    torch.manual_seed(3)
    sizes = [100, 0, 300, 128]
    padded, offs = _segments(sizes)
    rows = sum(padded)
    m, n = 256, 384
    a = torch.zeros(rows, m, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros(rows, n, device=DEV, dtype=torch.bfloat16)
    for s, o in zip(sizes, offs):
        a[o:o + s] = torch.randn(s, m, device=DEV, dtype=torch.bfloat16)
        b[o:o + s] = torch.randn(s, n, device=DEV, dtype=torch.bfloat16)
    out = torch.full((len(sizes), m, n), float("nan"), device=DEV, dtype=torch.float32)
    ops.ext().grouped_gemm_k(a, b, torch.tensor(offs, dtype=torch.int32, device=DEV),
                             torch.tensor(padded, dtype=torch.int32, device=DEV), out, False)
    for g, (s, o, p) in enumerate(zip(sizes, offs, padded)):
        ref = a[o:o + p].float().t() @ b[o:o + p].float() if p else torch.zeros(m, n, device=DEV)
        assert torch.isfinite(out[g]).all()
        if p:
            assert _rel(out[g], ref) < 1e-5
        else:
            assert out[g].abs().max().item() == 0


def test_linear_autograd():
    torch.manual_seed(4)
    x = torch.randn(3, 70, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(384, 256, device=DEV, dtype=torch.bfloat16) * 0.05).requires_grad_()
    y = G.linear(x, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = F.linear(xr, wr)
    yr.backward(gy.float())
    assert _rel(y, yr) < 5e-3
    assert _rel(x.grad, xr.grad) < 5e-3
    assert _rel(w.grad, wr.grad) < 5e-3


@pytest.mark.parametrize("h", [2048, 128, 5120, 264])
def test_rmsnorm(h):
    torch.manual_seed(5)
    x = torch.randn(67, h, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(h, device=DEV, dtype=torch.bfloat16)).requires_grad_()
    y = N.rms_norm(x, w, 1e-6)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = wr * (xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6))
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-2


def test_qk_norm_rope():
    torch.manual_seed(6)
    hq, hkv, t = 4, 2, 50
    qkv = torch.randn(t, (hq + 2 * hkv) * 128, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    wq = (1 + 0.1 * torch.randn(128, device=DEV, dtype=torch.bfloat16)).requires_grad_()
    wk = (1 + 0.1 * torch.randn(128, device=DEV, dtype=torch.bfloat16)).requires_grad_()
    pos = torch.arange(t, device=DEV) * 37
    freqs = R.inv_freq(128, 1e6, DEV)
    q, k, v = R.qk_norm_rope(qkv, wq, wk, pos, freqs, hq, hkv, 1e-6)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q.float() * gq.float()).sum().add((k.float() * gk.float()).sum()).add((v.float() * gv.float()).sum()).backward()
    qkv_r = qkv.detach().float().requires_grad_()
    wq_r, wk_r = wq.detach().float().requires_grad_(), wk.detach().float().requires_grad_()
    qr, kr, vr = R.qk_norm_rope_reference(qkv_r, wq_r, wk_r, pos, freqs, hq, hkv, 1e-6)
    (qr * gq.float()).sum().add((kr * gk.float()).sum()).add((vr * gv.float()).sum()).backward()
    assert _rel(q, qr) < 1e-2 and _rel(k, kr) < 1e-2 and _rel(v, vr) == 0
    assert _rel(qkv.grad, qkv_r.grad) < 1e-2
    assert _rel(wq.grad, wq_r.grad) < 1e-2 and _rel(wk.grad, wk_r.grad) < 1e-2


def test_rope_interleaved():
    torch.manual_seed(7)
    x = torch.randn(33, 4, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    pos = torch.arange(33, device=DEV)
    freqs = R.inv_freq(32, 10000.0, DEV)
    y = R.rope_interleaved(x, pos, freqs, 32)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    yr = R.rope_interleaved_reference(xr, pos, freqs, 32)
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2 and _rel(x.grad, xr.grad) < 1e-2
    back = R.rope_interleaved(y.detach(), pos, freqs, 32, inverse=True)
    assert _rel(back, x.detach()) < 2e-2


@pytest.mark.parametrize("func,e,k,bias", [("softmax", 128, 8, False), ("sqrtsoftplus", 384, 6, True),
                                           ("sigmoid", 64, 4, True)])
def test_router(func, e, k, bias):
    torch.manual_seed(8)
    t = 300
    logits = torch.randn(t, e, device=DEV, dtype=torch.float32, requires_grad=True)
    b = torch.randn(e, device=DEV) * 0.1 if bias else None
    aux = RT.AuxGradient()
    aux.set(torch.rand(e, device=DEV) * 1e-3)
    ids, w = RT.route(logits, k, func=func, bias=b, normalize=True, norm_eps=1e-20 if bias else 0.0,
                      scale=1.5, aux=aux)
    gw = torch.randn_like(w)
    w.backward(gw)
    lr = logits.detach().clone().requires_grad_()
    lr2 = RT._AuxHook.apply(lr, aux)
    ids_r, w_r = RT.route_reference(lr2, b, k, func, True, 1e-20 if bias else 0.0, 1.5)
    w_r.backward(gw)
    assert torch.equal(ids.long().sort(-1).values, ids_r.long().sort(-1).values)
    assert _rel(w.gather(-1, ids.long().argsort(-1)), w_r.gather(-1, ids_r.long().argsort(-1))) < 1e-5
    assert _rel(logits.grad, lr.grad) < 1e-4


def test_moe_gather_combine_swiglu():
    torch.manual_seed(9)
    t, h, e, k, inter = 200, 256, 8, 2, 192
    x = torch.randn(t, h, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    ids = torch.stack([torch.randperm(e, device=DEV)[:k] for _ in range(t)]).to(torch.int32)
    weights = torch.rand(t, k, device=DEV, requires_grad=True)
    routing = M.build_routing(ids, e)
    w1 = (torch.randn(e, 2 * inter, h, device=DEV, dtype=torch.bfloat16) * 0.05).requires_grad_()
    w2 = (torch.randn(e, h, inter, device=DEV, dtype=torch.bfloat16) * 0.05).requires_grad_()
    rows = M.gather(x, routing)
    gu = G.grouped_linear(rows, w1, routing.offsets, routing.rows)
    act = M.swiglu(gu)
    y = G.grouped_linear(act, w2, routing.offsets, routing.rows)
    out = M.combine(y, routing, weights)
    g = torch.randn_like(out)
    out.backward(g)
    # reference: per-token loop in fp32
    xr = x.detach().float().requires_grad_()
    wr = weights.detach().clone().requires_grad_()
    w1r, w2r = w1.detach().float().requires_grad_(), w2.detach().float().requires_grad_()
    outs = []
    for slot in range(k):
        eid = ids[:, slot].long()
        gate_up = torch.einsum("th,tnh->tn", xr, w1r[eid])
        gate, up = gate_up.chunk(2, dim=-1)
        hmid = F.silu(gate) * up
        outs.append(torch.einsum("ti,thi->th", hmid, w2r[eid]) * wr[:, slot:slot + 1])
    ref = sum(outs)
    ref.backward(g.float())
    assert _rel(out, ref) < 2e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(weights.grad, wr.grad) < 2e-2
    assert _rel(w1.grad, w1r.grad) < 2e-2
    assert _rel(w2.grad, w2r.grad) < 2e-2


def test_linear_cross_entropy():
    torch.manual_seed(10)
    t, h, v = 300, 256, 1000
    hidden = torch.randn(t, h, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(v, h, device=DEV, dtype=torch.bfloat16) * 0.05).requires_grad_()
    tgt = torch.randint(0, v, (t,), device=DEV)
    tgt[:50] = -100
    loss = ops.linear_cross_entropy(hidden, w, tgt, chunk=128)
    (loss * 0.5).backward()
    hr, wr = hidden.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    lr = F.cross_entropy(hr @ wr.t(), tgt, ignore_index=-100, reduction="sum")
    (lr * 0.5).backward()
    assert abs(loss.item() - lr.item()) / lr.item() < 1e-2
    assert _rel(hidden.grad, hr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2


def test_token_log_probs():
    torch.manual_seed(11)
    logits = torch.randn(40, 500, device=DEV, dtype=torch.float32, requires_grad=True)
    tgt = torch.randint(0, 500, (40,), device=DEV)
    lp = ops.token_log_probs(logits, tgt, 0.7)
    g = torch.randn_like(lp)
    lp.backward(g)
    lr = logits.detach().clone().requires_grad_()
    ref = F.log_softmax(lr / 0.7, -1).gather(-1, tgt[:, None]).squeeze(-1)
    ref.backward(g)
    assert _rel(lp, ref) < 1e-5 and _rel(logits.grad, lr.grad) < 1e-4


@pytest.mark.parametrize("moment_dtype", [torch.float32, torch.bfloat16])
def test_adamw(moment_dtype):
    torch.manual_seed(12)
    n = 10000
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    master = p.clone()
    m = torch.zeros(n, device=DEV, dtype=moment_dtype)
    v = torch.zeros(n, device=DEV, dtype=moment_dtype)
    out = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        ops.ext().adamw_step(master, g, m, v, out, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, 1.0, None)
        ref.grad = g.clone()
        opt.step()
    tol = 1e-6 if moment_dtype == torch.float32 else 1e-4
    assert (master - ref.detach()).abs().max().item() < tol
    assert _rel(out, ref.detach()) < 1e-2


def test_gemm_from_worker_thread():
    import threading

    a = torch.randn(256, 128, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(384, 128, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(256, 384, device=DEV, dtype=torch.float32)
    errors = []

    def work():
        try:
            ops.ext().gemm(a, b, out, False, False, False)
            torch.cuda.synchronize()
        except Exception as error:  # pragma: no cover
            errors.append(error)

    thread = threading.Thread(target=work)
    thread.start()
    thread.join()
    assert not errors
    assert _rel(out, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("n,k,e", [(67, 2, 8), (5000, 8, 16), (3000, 8, 128), (1, 1, 4)])
def test_moe_route_plan_matches_torch(n, k, e):
    torch.manual_seed(11)
    ids = torch.randint(-1, e, (n, k), dtype=torch.int32)
    ref = M.build_routing(ids, e)  # CPU: torch stable sort
    got = M.build_routing(ids.to(DEV), e)
    assert got.capacity == ref.capacity
    for name in ("route_rows", "src", "offsets", "rows", "counts", "total"):
        assert torch.equal(getattr(got, name).cpu(), getattr(ref, name)), name


def test_moe_route_plan_slabs():
    torch.manual_seed(12)
    slab, k, e = 64, 4, 8
    ids = torch.randint(0, e, (3 * slab, k), dtype=torch.int32)
    counts = torch.tensor([10, 0, 64], dtype=torch.int32)
    ref = M.build_routing(ids, e, slab_counts=counts, slab=slab)
    got = M.build_routing(ids.to(DEV), e, slab_counts=counts.to(DEV), slab=slab)
    for name in ("route_rows", "src", "offsets", "rows", "counts", "total"):
        assert torch.equal(getattr(got, name).cpu(), getattr(ref, name)), name
    assert (got.route_rows.cpu()[10:slab] == -1).all()


def test_ep_dest_plan():
    torch.manual_seed(13)
    t, k, ranks, per = 3000, 8, 8, 16
    ids = torch.randint(0, ranks * per, (t, k), dtype=torch.int32, device=DEV)
    dest, slot, counts = ops.ext().ep_dest_plan(ids, per, ranks)
    want = torch.zeros(t, ranks, dtype=torch.bool, device=DEV)
    want.scatter_(1, (ids // per).long(), True)
    assert torch.equal(dest.bool(), want)
    assert torch.equal(slot, (torch.cumsum(want.int(), 0) - 1).int())
    assert torch.equal(counts, want.sum(0).int())


def test_fp4_dequant_matches_torch():
    from tiny_dsv41_b200.ops.fp4 import dequantize_fp4
    from tiny_dsv41_b200.utils.quant import quantize_fp4_rows

    torch.manual_seed(14)
    w = torch.randn(96, 256) * 0.05
    packed, scale = quantize_fp4_rows(w)
    codes, scales = packed.view(torch.uint8), scale.view(torch.uint8)
    ref = dequantize_fp4(codes, scales)  # CPU restatement
    got = dequantize_fp4(codes.to(DEV), scales.to(DEV))
    assert torch.equal(got.cpu(), ref)


def test_frozen_fp4_grouped_linear_grad():
    from tiny_dsv41_b200.ops.fp4 import dequantize_fp4, fp4_grouped_linear
    from tiny_dsv41_b200.utils.quant import quantize_fp4_rows

    torch.manual_seed(15)
    e, n, k, per = 4, 256, 512, 128
    packed, scale = quantize_fp4_rows(torch.randn(e * n, k) * 0.05)
    codes = packed.view(torch.uint8).view(e, n, k // 2).to(DEV)
    scales = scale.view(torch.uint8).view(e, n, k // 32).to(DEV)
    x = torch.randn(e * per, k, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    off = torch.arange(e, device=DEV, dtype=torch.int32) * per
    rows = torch.full((e,), per, device=DEV, dtype=torch.int32)
    y = fp4_grouped_linear(x, codes, scales, off, rows, n)
    g = torch.randn_like(y)
    y.backward(g)
    w = dequantize_fp4(codes, scales).float()
    xr = x.detach().float().requires_grad_()
    yr = torch.cat([xr[i * per:(i + 1) * per] @ w[i].t() for i in range(e)])
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2


def test_fp4_grouped_gemm_converts_codes_exactly():
    """A one-hot activation picks single weight values out of the packed GEMM, so every E2M1 code
    times every E8M0 scale in range must come back bit-exact (forward: K-major weight tiles; input
    gradient: N-major tiles)."""
    from tiny_dsv41_b200.ops.fp4 import dequantize_fp4

    torch.manual_seed(16)
    n, k = 384, 128
    codes = torch.randint(0, 256, (1, n, k // 2), dtype=torch.uint8)
    scales = torch.randint(2, 251, (1, n, k // 32), dtype=torch.uint8)
    want = dequantize_fp4(codes, scales)[0]  # CPU restatement, [n, k]
    codes, scales = codes.to(DEV), scales.to(DEV)
    off = torch.zeros(1, device=DEV, dtype=torch.int32)
    rows = torch.full((1,), 128, device=DEV, dtype=torch.int32)
    eye = torch.eye(128, k, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(128, n, device=DEV, dtype=torch.bfloat16)
    ops.ext().fp4_grouped_gemm(eye, codes, scales, off, rows, out, False, 128)
    assert torch.equal(out.cpu(), want.t()[:128])
    # input gradient: codes [G, K = n, N = k] read N-major; a one-hot dy row picks weight row r
    dy = torch.eye(128, n, device=DEV, dtype=torch.bfloat16)
    dx = torch.empty(128, k, device=DEV, dtype=torch.bfloat16)
    ops.ext().fp4_grouped_gemm(dy, codes, scales, off, rows, dx, True, 128)
    assert torch.equal(dx.cpu(), want[:128])


@pytest.mark.parametrize("n,k", [(384, 256), (192, 320), (2048, 512)])
def test_fp4_grouped_gemm_ragged_groups(n, k, monkeypatch):
    """Uneven and empty expert groups, an N tail inside a tile, both tile widths; the packed path
    never expands the weight (the dequantisation kernel is not called)."""
    from tiny_dsv41_b200.ops import fp4 as F4
    from tiny_dsv41_b200.utils.quant import quantize_fp4_rows

    torch.manual_seed(17)
    sizes = [256, 0, 128, 384, 128]
    e = len(sizes)
    packed, scale = quantize_fp4_rows(torch.randn(e * n, k) * 0.05)
    codes = packed.view(torch.uint8).view(e, n, k // 2).to(DEV)
    scales = scale.view(torch.uint8).view(e, n, k // 32).to(DEV)
    w = F4.dequantize_fp4(codes, scales).float()
    starts = [sum(sizes[:i]) for i in range(e)]
    total = sum(sizes)
    x = torch.randn(total, k, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    off = torch.tensor(starts, device=DEV, dtype=torch.int32)
    rows = torch.tensor(sizes, device=DEV, dtype=torch.int32)

    def no_expansion(*_):
        raise AssertionError("the packed GEMM expanded the weight")

    monkeypatch.setattr(F4, "dequantize_fp4", no_expansion)
    y = F4.fp4_grouped_linear(x, codes, scales, off, rows, n)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    yr = torch.cat([xr[s0:s0 + c] @ w[i].t() for i, (s0, c) in enumerate(zip(starts, sizes))])
    yr.backward(g.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2


def test_bitwise_determinism_30_runs():
    """Fixed-order reductions: repeated launches give identical bits (combine, RMSNorm weight
    gradient, grouped weight-gradient GEMM, routing plan)."""
    torch.manual_seed(16)
    t, k, e, h = 700, 8, 16, 512
    ids = torch.randint(0, e, (t, k), dtype=torch.int32, device=DEV)
    routing = M.build_routing(ids, e)
    rows = torch.randn(routing.capacity, h, device=DEV, dtype=torch.bfloat16)
    w = torch.rand(t, k, device=DEV)
    x = torch.randn(t, h, device=DEV, dtype=torch.bfloat16)
    nw = torch.ones(h, device=DEV, dtype=torch.bfloat16)
    dy = torch.randn_like(x)
    _, rstd = ops.ext().rmsnorm_fwd(x, nw, 1e-6)
    gu = torch.randn(routing.capacity, 256, device=DEV, dtype=torch.bfloat16)
    first = None
    for _ in range(30):
        r = M.build_routing(ids, e)
        out = ops.ext().moe_combine(rows, r.route_rows, w)
        _, dw = ops.ext().rmsnorm_bwd(dy, x, nw, rstd, True)
        gw = torch.empty(e, 256, h, device=DEV, dtype=torch.bfloat16)
        ops.ext().grouped_gemm_k(gu, rows, r.offsets, r.rows, gw, False)
        cur = (r.route_rows.clone(), out.clone(), dw.clone(), gw.clone())
        if first is None:
            first = cur
        else:
            assert all(torch.equal(a, b) for a, b in zip(first, cur))
