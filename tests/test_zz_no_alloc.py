"""The allocation-free C entry point libra_rmsnorm_bwd_noalloc (ctypes) against
the torch-facing rmsnorm_bwd, on two calls in a row."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from libra_b200 import ops

    lib = ctypes.CDLL(ops.ext().__file__)
    fn = lib.libra_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    err = lib.libra_rmsnorm_bwd_noalloc_error
    err.restype = ctypes.c_char_p
    return fn, err


@pytest.mark.parametrize("T,H", [(4097, 2560), (300, 512), (64, 8192), (4096, 32768)])
def test_noalloc_matches_rmsnorm_bwd(T, H):
    from libra_b200 import ops

    fn, err = _lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(T + H)
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    dy = torch.randn(T, H, device=dev, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).bfloat16()
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    dw_ref = torch.empty(H, device=dev, dtype=torch.float32)
    dx_ref = ops.ext().rmsnorm_bwd(dy, x, w, rstd, dw_ref, False, None)
    stream = torch.cuda.current_stream()
    for _ in range(2):
        dx = torch.full_like(x, float("nan"))
        dw = torch.full((H,), float("nan"), device=dev)
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), T, H, 0, 0,
                stream.cuda_stream)
        assert rc == 0, err()
        torch.cuda.synchronize()
        torch.testing.assert_close(dx.float(), dx_ref.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dw, dw_ref, rtol=1e-4, atol=1e-3)


def test_noalloc_accumulates_and_rejects_oversize():
    fn, err = _lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    T, H = 128, 1024
    x = torch.randn(T, H, device=dev).bfloat16()
    dy = torch.randn(T, H, device=dev).bfloat16()
    w = torch.ones(H, device=dev).bfloat16()
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    s = torch.cuda.current_stream().cuda_stream
    dx = torch.zeros_like(x)
    dw = torch.zeros(H, device=dev)
    args = (dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr())
    assert fn(*args, T, H, 1, 1, s) == 0, err()
    dx1, dw1 = dx.clone(), dw.clone()
    assert fn(*args, T, H, 1, 1, s) == 0, err()
    torch.cuda.synchronize()
    torch.testing.assert_close(dx.float(), 2 * dx1.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(dw, 2 * dw1, rtol=1e-5, atol=1e-5)
    assert fn(*args, T, 65536, 0, 0, s) == 2 and b"limit" in err()
    assert fn(*args, T, 1001, 0, 0, s) == 1
