"""The allocation-free weight-gradient entry point, called through its C symbol.

Callers that cannot allocate device memory while they run (plugins inside
another runtime's memory budget, real-time loops, C hosts without PyTorch's
allocator) use ``cfb_weight_grad_noalloc``: its fp32 accumulator is a fixed
array inside the library.  Its results must match the framework's regular
weight-gradient path, call after call.  This file is collected last so that a
run stopping at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ELEMS = 4 * 1024 * 1024


def _entry():
    import complexity_framework_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.cfb_weight_grad_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _status():
    import complexity_framework_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.cfb_weight_grad_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    out = (ctypes.c_int * 4)(-1, -1, -1, -1)
    rc = fn(out, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, list(out)


def _call(fn, dy, x, out):
    T, N = dy.shape
    K = x.shape[1]
    return fn(dy.data_ptr(), x.data_ptr(), T, N, K, out.data_ptr(),
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _check(out, ref, tol=2e-2):
    err = (out.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err / scale < tol, f"max rel err {err / scale:.3e}"


def test_noalloc_weight_grad_matches_existing_entry_point():
    from complexity_framework_b200.ops.fused import gemm_tn

    fn = _entry()
    g = torch.Generator().manual_seed(0)
    for T, N, K in ((4096, 896, 1152), (2048, 640, 256)):   # two calls in a row
        dy = torch.randn(T, N, generator=g).cuda().bfloat16()
        x = torch.randn(T, K, generator=g).cuda().bfloat16()
        out = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        assert _call(fn, dy, x, out) == 0
        ref = gemm_tn(dy, x)                      # the framework's regular path
        torch.cuda.synchronize()
        _check(out, ref)
        _check(out, dy.float().t() @ x.float())   # and the fp32 definition
        # no bounded wait of the GEMM timed out, and the status word reads clear
        assert _status() == (0, [0, 0, 0, 0])


def test_noalloc_rejects_oversized_output():
    fn = _entry()
    dy = torch.zeros(64, 4096, device="cuda", dtype=torch.bfloat16)
    x = torch.zeros(64, 2048, device="cuda", dtype=torch.bfloat16)   # 4096*2048 > max
    out = torch.empty(4096, 2048, device="cuda", dtype=torch.bfloat16)
    assert 4096 * 2048 > MAX_ELEMS
    assert _call(fn, dy, x, out) == -1
