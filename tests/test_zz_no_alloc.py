"""The allocation-free RMSNorm backward, called through its exported C symbol.

It must match the PyTorch-facing ``rmsnorm_bwd`` entry point on two calls in a row that share the
library's one scratch array (the second call smaller than the first, so stale scratch contents
would show), and reject a hidden size beyond the array's capacity before touching the GPU.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_HIDDEN = 8192
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


def test_noalloc_matches_rmsnorm_bwd_twice():
    from tiny_dsv41_b200.ops._ext import ext

    fn = _entry()
    stream = torch.cuda.current_stream()
    # first call: more 32-row chunks than scratch rows (128), so blocks loop; second call smaller
    for rows, h, wdtype, seed in ((4133, 2048, torch.float32, 0), (67, 1024, torch.bfloat16, 1)):
        dy, x, w, rstd = _case(rows, h, wdtype, seed)
        dx = torch.empty_like(x)
        dw = torch.empty(h, device="cuda", dtype=torch.float32)
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), int(wdtype == torch.bfloat16), rstd.data_ptr(),
                dx.data_ptr(), dw.data_ptr(), rows, h, stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        dx_ref, dw_ref = ext().rmsnorm_bwd(dy, x, w, rstd, True)
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 1e-2, (rows, h)
        assert _rel(dw, dw_ref) < 1e-2, (rows, h)


def test_noalloc_rejects_oversize_hidden():
    fn = _entry()
    rc = fn(None, None, None, 0, None, None, None, 8, MAX_HIDDEN + 8, None)
    assert rc == ETOOBIG
