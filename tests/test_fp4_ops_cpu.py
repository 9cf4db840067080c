"""The frozen MXFP4 grouped linear on CPU (the path the packed tcgen05 GEMM replaces on GPUs):
forward and input gradient against an explicit dequantise-then-matmul in fp32."""

import torch

from tiny_dsv41_b200.ops.fp4 import dequantize_fp4, fp4_grouped_linear
from tiny_dsv41_b200.utils.quant import quantize_fp4_rows


def test_fp4_grouped_linear_cpu_forward_and_input_gradient():
    torch.manual_seed(0)
    sizes = [128, 0, 256]
    e, n, k = len(sizes), 96, 64
    packed, scale = quantize_fp4_rows(torch.randn(e * n, k) * 0.05)
    codes = packed.view(torch.uint8).view(e, n, k // 2)
    scales = scale.view(torch.uint8).view(e, n, k // 32)
    w = dequantize_fp4(codes, scales).float()
    starts = [sum(sizes[:i]) for i in range(e)]
    x = torch.randn(sum(sizes), k, requires_grad=True)
    y = fp4_grouped_linear(x, codes, scales, torch.tensor(starts, dtype=torch.int32),
                           torch.tensor(sizes, dtype=torch.int32), n)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().clone().requires_grad_()
    yr = torch.cat([xr[s:s + c] @ w[i].t() for i, (s, c) in enumerate(zip(starts, sizes))])
    yr.backward(g)
    assert torch.allclose(y, yr, atol=1e-5, rtol=1e-5)
    assert torch.allclose(x.grad, xr.grad, atol=1e-5, rtol=1e-5)


def test_dequantize_fp4_every_code_and_scale_sign():
    """All 16 E2M1 codes at a few E8M0 scales, both nibbles: value = sign * mag * 2^(s - 127)."""
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    codes = torch.arange(256, dtype=torch.uint8).view(8, 32)  # every byte once
    scales = torch.tensor([[100], [120], [127], [130], [140], [110], [125], [128]], dtype=torch.uint8)
    out = dequantize_fp4(codes, scales).float()
    for r in range(8):
        for c in range(64):
            byte = int(codes[r, c // 2])
            nib = byte & 0xF if c % 2 == 0 else byte >> 4
            want = (-1.0 if nib & 8 else 1.0) * mags[nib & 7] * 2.0 ** (int(scales[r, 0]) - 127)
            assert out[r, c].item() == want, (r, c, out[r, c].item(), want)
