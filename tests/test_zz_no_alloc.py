"""GPU: the allocation-free W8A8 entry point (dgx_gemm_w8a8_noalloc).

It is meant for callers that must not let a library allocate device memory
(their pool owns the whole budget, or their serving loop may not call
cudaMalloc). Through the C ABI it must give the same result as the
allocating entry point dgx_gemm_w8(mode=1), on two calls in a row (the fixed
scratch array is shared and keeps the previous call's contents), and refuse
problems larger than its fixed scratch.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process (the first
call sets up the array's device address).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _call_noalloc(lib, X, W, sc, b, Y):
    B, K = X.shape
    N = W.shape[0]
    return lib.dgx_gemm_w8a8_noalloc(X.data_ptr(), W.data_ptr(), sc.data_ptr(), b.data_ptr(), Y.data_ptr(), B, N, K,
                                     torch.cuda.current_stream().cuda_stream)


def _call_alloc(lib, X, W, sc, b, Y):
    B, K = X.shape
    N = W.shape[0]
    return lib.dgx_gemm_w8(X.data_ptr(), W.data_ptr(), sc.data_ptr(), b.data_ptr(), Y.data_ptr(), B, N, K, 1,
                           torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    assert lib.dgx_init(0) == _lib.DGX_OK
    # two calls in a row with different shapes and data: the second must not
    # see anything left over from the first in the shared scratch
    for call, (B, N, K) in enumerate([(256, 4096, 4096), (16, 1000, 4096)]):
        g = torch.Generator(device="cuda").manual_seed(11 + call)
        X = torch.randn(B, K, device="cuda", generator=g)
        W = torch.randint(-127, 128, (N, K), device="cuda", dtype=torch.int8, generator=g)
        sc = torch.rand(N, device="cuda", generator=g) * 9e-3 + 1e-3
        b = torch.randn(N, device="cuda", generator=g)
        Y_free = torch.empty(B, N, device="cuda")
        Y_ref = torch.empty(B, N, device="cuda")
        _lib.check(_call_noalloc(lib, X, W, sc, b, Y_free), "dgx_gemm_w8a8_noalloc")
        _lib.check(_call_alloc(lib, X, W, sc, b, Y_ref), "dgx_gemm_w8")
        _lib.check(lib.dgx_sync_check(torch.cuda.current_stream().cuda_stream), "dgx_sync_check")
        assert normwise(Y_free.cpu().numpy(), Y_ref.cpu().numpy()) < 1e-6, f"call {call}"


def test_noalloc_rejects_problems_beyond_its_scratch():
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    dummy = C.c_void_p(256)
    # B*K above 4,194,304 activations, and B above 4096 rows
    for B, K in ((1024, 8192), (4097, 16)):
        st = lib.dgx_gemm_w8a8_noalloc(dummy, dummy, dummy, None, dummy, B, 64, K, None)
        assert st == _lib.DGX_EINVAL
        assert b"exceeds the fixed scratch" in lib.dgx_last_error()
