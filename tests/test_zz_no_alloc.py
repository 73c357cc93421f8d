"""The allocation-free C entry point of the RMSNorm backward (fyb_rms_norm_bwd_noalloc).

It exists for callers that cannot allocate device memory (a foreign runtime that owns all device memory and passes
only input/output buffers, or a path where cudaMalloc's synchronisation is not allowed). The test calls it through
its exported C symbol, twice in a row (the static scratch array is reused and keeps the previous call's partials),
and compares both results with the library's regular entry point. This file sorts last so that a run stopping at
the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    import faster_yoco_b200._C as ext          # torch is imported first, so the library's dependencies resolve
    lib = ctypes.CDLL(ext.__file__)
    f = lib.fyb_rms_norm_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    err = lib.fyb_noalloc_strerror
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return ext, f, err


def rel(x, r):
    x, r = x.float(), r.float()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("M,N", [(2048, 3072), (37, 8192)])
def test_noalloc_rms_norm_bwd_matches_regular_entry_point(M, N):
    ext, f, err = _entry()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.manual_seed(M + N)
    x = torch.randn(M, N, device=dev, dtype=torch.bfloat16) * 2
    w = (torch.rand(N, device=dev) + 0.5).to(torch.bfloat16)
    _, rstd = ext.rms_norm_fwd(x, w, 1e-5)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        dy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        dx_ref, dw_ref = ext.rms_norm_bwd(dy, x, w, rstd)
        dx = torch.empty_like(x)
        dw = torch.empty(N, device=dev, dtype=torch.bfloat16)
        rc = f(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), M, N,
               stream)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert rel(dx, dx_ref) < 1e-2, call
        assert rel(dw, dw_ref) < 2e-2, call


def test_noalloc_rejects_width_beyond_scratch():
    ext, f, err = _entry()
    dev = torch.device("cuda", 0)
    M, N = 4, 8200
    x = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    w = torch.ones(N, device=dev, dtype=torch.bfloat16)
    rstd = torch.ones(M, device=dev)
    dx = torch.empty_like(x)
    dw = torch.empty(N, device=dev, dtype=torch.bfloat16)
    rc = f(x.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), M, N,
           torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"8192" in err(rc)
