"""The allocation-free RMSNorm backward, called through its exported C symbol.

It must match the PyTorch-facing ``rmsnorm_bwd`` entry point on calls in a row that share the
library's one scratch array (later calls smaller than earlier ones, so stale scratch contents
would show), agree with a float64 autograd restatement, skip the weight gradient when ``dw`` is
NULL, and reject a hidden size beyond the array's capacity or a misaligned row pointer before
touching the GPU.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_HIDDEN = 8192
EINVAL = 1
ETOOBIG = 2


def _entry():
    from tiny_dsv41_b200.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    fn = lib.tdsv_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return fn


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _case(rows, h, wdtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, h, device="cuda", dtype=torch.bfloat16, generator=g)
    dy = torch.randn(rows, h, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(wdtype)
    rstd = torch.rsqrt(x.float().square().mean(-1) + 1e-6)
    return dy, x, w, rstd


def _call(fn, dy, x, w, rstd, dx, dw, rows, h):
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), int(w.dtype == torch.bfloat16), rstd.data_ptr(),
              dx.data_ptr(), None if dw is None else dw.data_ptr(), rows, h, torch.cuda.current_stream().cuda_stream)


# (rows, h, weight dtype, seed), run back to back on the one scratch array: the first has more 32-row
# chunks than scratch rows (128), so blocks loop; h = 8192 fills all four register passes of 2048
# columns, h = 3072 stops inside the second; later calls are smaller than earlier ones, so stale
# scratch contents would show
CASES = ((4133, 2048, torch.float32, 0), (67, 1024, torch.bfloat16, 1), (1001, 8192, torch.float32, 2),
         (333, 3072, torch.bfloat16, 3), (77, 8192, torch.bfloat16, 4), (333, 3072, torch.float32, 5))


def test_noalloc_matches_rmsnorm_bwd_in_sequence():
    from tiny_dsv41_b200.ops._ext import ext

    fn = _entry()
    for rows, h, wdtype, seed in CASES:
        dy, x, w, rstd = _case(rows, h, wdtype, seed)
        dx = torch.empty_like(x)
        dw = torch.empty(h, device="cuda", dtype=torch.float32)
        assert _call(fn, dy, x, w, rstd, dx, dw, rows, h) == 0
        torch.cuda.synchronize()
        dx_ref, dw_ref = ext().rmsnorm_bwd(dy, x, w, rstd, True)
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 1e-2, (rows, h)
        assert _rel(dw, dw_ref) < 1e-2, (rows, h)


def test_noalloc_matches_float64_autograd():
    """Independent oracle: float64 autograd of y = w * (x * rsqrt(mean(x^2) + eps)) for dx, and the
    float64 sum of dy * bf16(x * rstd) for dw (the forward stores the normalised row in bf16)."""
    fn = _entry()
    rows, h = 515, 3072
    dy, x, w, rstd = _case(rows, h, torch.float32, 7)
    dx = torch.empty_like(x)
    dw = torch.empty(h, device="cuda", dtype=torch.float32)
    assert _call(fn, dy, x, w, rstd, dx, dw, rows, h) == 0
    torch.cuda.synchronize()
    x64 = x.double().requires_grad_(True)
    y = w.double() * (x64 * torch.rsqrt(x64.square().mean(-1, keepdim=True) + 1e-6))
    (y * dy.double()).sum().backward()
    dw64 = (dy.double() * (x.float() * rstd[:, None]).to(torch.bfloat16).double()).sum(0)
    assert _rel(dx, x64.grad) < 1e-2
    assert _rel(dw, dw64) < 1e-3


def test_noalloc_without_weight_gradient():
    from tiny_dsv41_b200.ops._ext import ext

    fn = _entry()
    rows, h = 300, 8192
    dy, x, w, rstd = _case(rows, h, torch.bfloat16, 8)
    dx = torch.empty_like(x)
    assert _call(fn, dy, x, w, rstd, dx, None, rows, h) == 0
    torch.cuda.synchronize()
    dx_ref, _ = ext().rmsnorm_bwd(dy, x, w, rstd, True)
    assert _rel(dx, dx_ref) < 1e-2


def test_noalloc_rejects_misaligned_rows_before_launching():
    fn = _entry()
    rows, h = 16, 1024
    dy, x, w, rstd = _case(rows, h, torch.float32, 9)
    dx = torch.empty_like(x)
    dw = torch.empty(h, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(dy.data_ptr() + 2, x.data_ptr(), w.data_ptr(), 0, rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, h,
            stream)
    assert rc == EINVAL
    rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), 0, rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, 1020,
            stream)
    assert rc == EINVAL  # h not a multiple of 8


def test_noalloc_rejects_oversize_hidden():
    fn = _entry()
    rc = fn(None, None, None, 0, None, None, None, 8, MAX_HIDDEN + 8, None)
    assert rc == ETOOBIG
