"""Single-GPU microbenchmarks of the hot kernels, reported against the measured roofline.

    python bench_kernels.py                      # every case, JSON lines
    python bench_kernels.py --case grouped_fwd   # one case
    python bench_kernels.py --case grouped_fwd --once   # warm up, then exactly one launch (for ncu)

Each case times its kernel with CUDA events on the launching stream after warm-up (inputs are
larger than the 126 MB L2 unless noted) and reports achieved TFLOP/s or GB/s and the fraction of
``MEASURED_PEAKS.json`` (cuBLAS bf16 burst / copy bandwidth measured on this hardware); GEMM
cases also time ``torch.matmul`` (cuBLAS) on the same operands, attention cases PyTorch's
scaled-dot-product attention (cuDNN on B200) on the same q / k / v.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"tflops": p["bf16_tflops"], "gbs": p["hbm_gbs"], "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1590.0, "gbs": 6650.0, "source": "fallback"}


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def cases():
    from tiny_dsv41_b200 import ops

    C = ops.ext()
    dev = "cuda"
    bf = torch.bfloat16

    def dense(m, n, k):
        a = torch.randn(m, k, device=dev, dtype=bf)
        b = torch.randn(n, k, device=dev, dtype=bf)
        out = torch.empty(m, n, device=dev, dtype=bf)
        return (lambda: C.gemm(a, b, out, False, False, False)), (lambda: torch.matmul(a, b.t())), 2 * m * n * k, None

    def grouped(kind, experts=16, per=2048, h=2048, inter=768):
        rows = experts * per
        off = torch.arange(experts, device=dev, dtype=torch.int32) * per
        size = torch.full((experts,), per, device=dev, dtype=torch.int32)
        x = torch.randn(rows, h, device=dev, dtype=bf)
        w1 = torch.randn(experts, 2 * inter, h, device=dev, dtype=bf) * 0.02
        gu = torch.randn(rows, 2 * inter, device=dev, dtype=bf)
        flops = 2 * rows * 2 * inter * h
        if kind == "fwd":
            out = torch.empty(rows, 2 * inter, device=dev, dtype=bf)
            ends = torch.cumsum(size, 0, dtype=torch.int32)
            w1t = w1.transpose(1, 2)
            return ((lambda: C.grouped_gemm_m(x, w1, off, size, out, False, rows)),
                    (lambda: torch._grouped_mm(x, w1t, offs=ends)), flops, None)
        if kind == "dx":
            out = torch.empty(rows, h, device=dev, dtype=bf)
            return (lambda: C.grouped_gemm_m(gu, w1, off, size, out, True, rows)), None, flops, None
        out = torch.empty(experts, 2 * inter, h, device=dev, dtype=bf)
        return (lambda: C.grouped_gemm_k(gu, x, off, size, out, False)), None, flops, None

    def adamw(n=256 << 20):
        p = torch.randn(n, device=dev)
        g = torch.randn(n, device=dev, dtype=bf)
        m = torch.zeros(n, device=dev)
        v = torch.zeros(n, device=dev)
        out = torch.empty(n, device=dev, dtype=bf)
        step = (lambda: C.adamw_step(p, g, m, v, out, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, 1.0, None))
        return step, None, None, n * (4 + 2 + 4 + 4 + 4 + 4 + 4 + 2)

    def swiglu(rows=65536, inter=768):
        gu = torch.randn(rows, 2 * inter, device=dev, dtype=bf)
        return (lambda: C.swiglu_fwd(gu, None, False, 0.0, None)), None, None, rows * inter * 2 * 3

    def rmsnorm(rows=32768, h=4096):
        x = torch.randn(rows, h, device=dev, dtype=bf)
        w = torch.ones(h, device=dev, dtype=bf)
        return (lambda: C.rmsnorm_fwd(x, w, 1e-6)), None, None, rows * h * 2 * 2

    def attention(kind, batch=1, seq=4096, heads=32, kv_heads=4):
        # Qwen3-30B-A3B attention shape; causal FLOPs = half of the dense 4 * B * H * L^2 * D
        import torch.nn.functional as F

        q = torch.randn(batch, seq, heads, 128, device=dev, dtype=bf)
        k = torch.randn(batch, seq, kv_heads, 128, device=dev, dtype=bf)
        v = torch.randn(batch, seq, kv_heads, 128, device=dev, dtype=bf)
        fwd_flops = 2 * batch * heads * seq * seq * 128
        qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if kind == "fwd":
            def sdpa():
                return F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
            return (lambda: C.attn_fwd(q, k, v)), sdpa, fwd_flops, None
        out, lse = C.attn_fwd(q, k, v)
        dout = torch.randn_like(q)
        qr, kr, vr = (t.detach().requires_grad_() for t in (qh, kh, vh))
        ref_out = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True, enable_gqa=True)
        dref = dout.transpose(1, 2)

        def sdpa_bwd():
            return torch.autograd.grad(ref_out, (qr, kr, vr), dref, retain_graph=True)
        return (lambda: C.attn_bwd(dout, q, k, v, out, lse)), sdpa_bwd, int(2.5 * fwd_flops), None

    def index_scores(batch=1, seq=4096, heads=32, dim=128, ratio=4):
        # DeepSeek-V4-Flash indexer shape: 32 heads x 128, one compressed key per `ratio` tokens;
        # FLOPs of the dense score tile (queries x visible-key window x heads x dim)
        keys_len = seq // ratio
        q = torch.randn(batch, seq, heads, dim, device=dev, dtype=bf)
        k = torch.randn(batch, keys_len, dim, device=dev, dtype=bf)
        w = torch.randn(batch, seq, heads, device=dev) * heads ** -0.5
        starts = torch.zeros(batch, seq, dtype=torch.int32, device=dev)
        ends = ((torch.arange(seq, device=dev) + 1) // ratio).clamp_min(1).to(torch.int32).expand(batch, seq).contiguous()
        width = keys_len
        flops = 2 * batch * seq * width * heads * dim
        return (lambda: C.index_scores(q, k, w, starts, ends, width, None)), None, flops, None

    def sparse_attention(kind, batch=1, seq=4096, heads=64, dim=512, window=128, selected=512, comp_ratio=4):
        # DeepSeek-V4-Flash-like sparse attention: 64 heads share one 512-wide latent KV row per key;
        # each token sees its 128 window keys and 512 selected compressed keys (plus the sink).
        # FLOPs: QK^T and PV per (token, head, key); the reference is the gathered PyTorch
        # restatement (einsum on gathered [B, L, keys, D] tensors) timed on the same inputs.
        from tiny_dsv41_b200.ops.sparse_attention import sparse_attention_reference

        comp_len = seq // comp_ratio
        q = torch.randn(batch, seq, heads, dim, device=dev, dtype=bf)
        kv = torch.randn(batch, seq, dim, device=dev, dtype=bf)
        comp = torch.randn(batch, comp_len, dim, device=dev, dtype=bf)
        pos = torch.arange(seq, device=dev).view(1, -1, 1)
        widx = (pos - window + 1 + torch.arange(window, device=dev).view(1, 1, -1))
        wmask = (widx >= 0).expand(batch, -1, -1).contiguous()
        widx = widx.clamp_min(0).expand(batch, -1, -1).contiguous()
        sel = torch.randint(0, comp_len, (batch, seq, selected), device=dev)
        sinks = torch.randn(heads, device=dev)
        keys = window + selected
        fwd_flops = 4 * batch * seq * heads * keys * dim
        if kind == "fwd":
            return ((lambda: C.sparse_attention_fwd(q, kv, widx, wmask, comp, sel, sinks)),
                    (lambda: sparse_attention_reference(q.transpose(1, 2), kv, widx, wmask, comp, sel, sinks)),
                    fwd_flops, None)
        out, lse = C.sparse_attention_fwd(q, kv, widx, wmask, comp, sel, sinks)
        dout = torch.randn_like(out)
        return ((lambda: C.sparse_attention_bwd(q, kv, widx, wmask, comp, sel, sinks, out, lse, dout)), None,
                int(2.5 * fwd_flops), None)

    def peer_update(n=256 * 1024 * 1024, moments=torch.bfloat16, blocks=1184):
        # the fused dense-sync kernel of parallel/peer_fsdp.py on one GPU (world 1: the peer
        # tables hold the local pools), one 256M-element unit with bf16 moments. Bytes per element:
        # gradient 2 + parameter 2 + master 8 + moments 8 (bf16, read and written) = 20.
        pool = torch.randn(n, device=dev, dtype=bf)
        grad = torch.randn(n, device=dev, dtype=bf)
        flags = torch.zeros(2, 1, dtype=torch.int32, device=dev)
        master = pool.float()
        m = torch.zeros(n, device=dev, dtype=moments)
        v = torch.zeros(n, device=dev, dtype=moments)
        tables = [torch.tensor([t.data_ptr()], dtype=torch.int64) for t in (grad, pool, flags)]
        epoch = [0]

        def step():
            epoch[0] += 1
            C.peer_update(tables[0], tables[1], tables[2], flags, 0, 0, epoch[0], 0, master, m, v, 0, 1e-4, 0.9,
                          0.95, 1e-8, 0.1, epoch[0], 1.0, None, None, blocks)
        return step, None, None, n * (2 + 2 + 8 + 2 * 2 * moments.itemsize)

    def fp4_grouped(kind, experts=48, per=512, n=4608, k=5120):
        # frozen MXFP4 experts at DSV4-Flash gate_up shapes for one EP8 rank (384 / 8 experts,
        # 4096 tokens x top-6 / 48 = 512 rows each), weight W [n, k] packed along k. The
        # comparison is the former path, which expanded the codes to a bf16 weight in HBM and ran
        # the bf16 grouped GEMM.
        rows_n, cols = (n, k) if kind == "fwd" else (k, n)  # output columns, contraction (dx reads W N-major)
        codes = torch.randint(0, 256, (experts, n, k // 2), device=dev, dtype=torch.uint8)
        scales = torch.randint(118, 130, (experts, n, k // 32), device=dev, dtype=torch.uint8)
        x = torch.randn(experts * per, cols, device=dev, dtype=bf)
        out = torch.empty(experts * per, rows_n, device=dev, dtype=bf)
        off = (torch.arange(experts, device=dev, dtype=torch.int32) * per).contiguous()
        cnt = torch.full((experts,), per, device=dev, dtype=torch.int32)
        b_mn = kind == "dx"

        def expand_then_gemm():
            w = C.fp4_dequant(codes, scales)
            C.grouped_gemm_m(x, w, off, cnt, out, b_mn, x.shape[0])
        return ((lambda: C.fp4_grouped_gemm(x, codes, scales, off, cnt, out, b_mn, x.shape[0])), expand_then_gemm,
                2 * experts * per * n * k, None)

    return {
        "peer_update": peer_update,
        "sparse_attn_fwd": lambda: sparse_attention("fwd"),
        "sparse_attn_bwd": lambda: sparse_attention("bwd"),
        "dense_lm_head": lambda: dense(4096, 151936, 2048),
        "dense_qkv": lambda: dense(4096, 5120, 2048),
        "dense_8192": lambda: dense(8192, 8192, 8192),
        "grouped_fwd": lambda: grouped("fwd"),
        "grouped_dx": lambda: grouped("dx"),
        "grouped_dw": lambda: grouped("dw"),
        # the Qwen3-30B-A3B step at EP2: 4096 tokens x top-8 per rank over 64 local experts
        "step_grouped_fwd": lambda: grouped("fwd", experts=64, per=512),
        "step_grouped_dx": lambda: grouped("dx", experts=64, per=512),
        "step_grouped_dw": lambda: grouped("dw", experts=64, per=512),
        "fp4_grouped_fwd": lambda: fp4_grouped("fwd"),
        "fp4_grouped_dx": lambda: fp4_grouped("dx"),
        "adamw": adamw,
        "swiglu": swiglu,
        "rmsnorm": rmsnorm,
        "attn_fwd": lambda: attention("fwd"),
        "attn_bwd": lambda: attention("bwd"),
        "index_scores": index_scores,
    }


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--case", default="all")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--once", action="store_true", help="warm up, then launch the case exactly once")
    args = p.parse_args(argv)
    peaks = _peaks()
    table = cases()
    names = list(table) if args.case == "all" else [args.case]
    for name in names:
        fn, ref, flops, nbytes = table[name]()
        if args.once:
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            fn()
            torch.cuda.synchronize()
            continue
        ms = _time(fn, args.iters)
        row = {"case": name, "ms": round(ms, 4)}
        if flops:
            row.update(tflops=round(flops / ms / 1e9, 1), frac_of_peak=round(flops / ms / 1e9 / peaks["tflops"], 3))
        if nbytes:
            row.update(gbs=round(nbytes / ms / 1e6, 1), frac_of_peak=round(nbytes / ms / 1e6 / peaks["gbs"], 3))
        if ref is not None:
            rms = _time(ref, args.iters)
            label = ("cudnn_sdpa" if name.startswith("attn") else "gathered_torch" if name.startswith("sparse")
                     else "expand_then_gemm" if name.startswith("fp4")
                     else "torch_grouped_mm" if "grouped" in name else "cublas")
            row.update({f"{label}_ms": round(rms, 4), f"{label}_tflops": round(flops / rms / 1e9, 1)})
        row["peak_source"] = peaks["source"]
        print(json.dumps(row), flush=True)
        del fn, ref
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
