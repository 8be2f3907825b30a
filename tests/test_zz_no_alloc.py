"""GPU: the allocation-free W8A8 entry point (dgx_gemm_w8a8_noalloc).

It is meant for callers that must not let a library allocate device memory
(their pool owns the whole budget, or their serving loop may not call
cudaMalloc). Through the C ABI it must give the same bits as the allocating
entry point dgx_gemm_w8(mode=1) on two calls in a row (the fixed scratch
array is shared and keeps the previous call's contents), match the oracle's
quantiser and exact int32 products, and refuse problems larger than its
fixed scratch.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process, and one test
runs it in a child process that never calls dgx_init.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, normwise

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


def _inputs(B, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(B, K, device="cuda", generator=g)
    W = torch.randint(-127, 128, (N, K), device="cuda", dtype=torch.int8, generator=g)
    sc = torch.rand(N, device="cuda", generator=g) * 9e-3 + 1e-3
    b = torch.randn(N, device="cuda", generator=g)
    return X, W, sc, b


# Consecutive calls with different shapes: the tensor-core route (K % 16 == 0),
# the SIMT route (K % 16 != 0, generic quantiser), and B*K exactly at the
# array's 4,194,304-activation limit.
SHAPES = [(256, 4096, 4096), (16, 1000, 4096), (8, 130, 1000), (1024, 512, 4096)]


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    assert lib.dgx_init(0) == _lib.DGX_OK
    for call, (B, N, K) in enumerate(SHAPES):
        X, W, sc, b = _inputs(B, N, K, 11 + call)
        Y_free = torch.full((B, N), float("nan"), device="cuda")
        Y_ref = torch.empty(B, N, device="cuda")
        _lib.check(_call_noalloc(lib, X, W, sc, b, Y_free), "dgx_gemm_w8a8_noalloc")
        _lib.check(_call_alloc(lib, X, W, sc, b, Y_ref), "dgx_gemm_w8")
        _lib.check(lib.dgx_sync_check(torch.cuda.current_stream().cuda_stream), "dgx_sync_check")
        # same kernels on the same data: the same bits
        assert torch.equal(Y_free, Y_ref), f"call {call} {(B, N, K)}"


def test_noalloc_matches_the_oracle(orc):
    """The int32 core and the quantiser, pinned once to the oracle's
    restatement: Y = bias + scale[n] * sx[b] * sum_k q[b,k] W[n,k]."""
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    for B, N, K in ((16, 384, 4096), (8, 130, 1000)):
        X, W, sc, b = _inputs(B, N, K, 5 + K)
        Y = torch.empty(B, N, device="cuda")
        _lib.check(_call_noalloc(lib, X, W, sc, b, Y), "dgx_gemm_w8a8_noalloc")
        _lib.check(lib.dgx_sync_check(torch.cuda.current_stream().cuda_stream), "dgx_sync_check")
        Xh, Wh, sch, bh = (t.cpu().numpy() for t in (X, W, sc, b))
        rXq, rsx = orc.quantize_rows(Xh)
        racc = orc.i8_gemm(rXq, Wh)
        ref = bh.astype(np.float64) + sch.astype(np.float64) * rsx.astype(np.float64)[:, None] * racc
        assert normwise(Y.cpu().numpy(), ref) < 1e-6, (B, N, K)


_CHILD = r"""
import sys, torch, numpy as np
sys.path.insert(0, sys.argv[1])
from dreamcompiler_b200 import _lib
lib = _lib.load()  # no dgx_init: the entry point must not need it
torch.cuda.set_device(0)
g = torch.Generator(device="cuda").manual_seed(3)
B, N, K = 64, 256, 2048
X = torch.randn(B, K, device="cuda", generator=g)
W = torch.randint(-127, 128, (N, K), device="cuda", dtype=torch.int8, generator=g)
sc = torch.rand(N, device="cuda", generator=g) * 9e-3 + 1e-3
b = torch.randn(N, device="cuda", generator=g)
s = torch.cuda.current_stream().cuda_stream
Ys = []
for _ in range(2):
    Y = torch.empty(B, N, device="cuda")
    _lib.check(lib.dgx_gemm_w8a8_noalloc(X.data_ptr(), W.data_ptr(), sc.data_ptr(), b.data_ptr(), Y.data_ptr(),
                                         B, N, K, s), "noalloc")
    Ys.append(Y)
torch.cuda.synchronize()
Yr = torch.empty(B, N, device="cuda")
_lib.check(lib.dgx_gemm_w8(X.data_ptr(), W.data_ptr(), sc.data_ptr(), b.data_ptr(), Yr.data_ptr(), B, N, K, 1, s),
           "w8")
_lib.check(lib.dgx_sync_check(s), "sync")
assert torch.equal(Ys[0], Yr) and torch.equal(Ys[1], Yr)
print("child ok")
"""


def test_noalloc_in_a_fresh_process_without_dgx_init():
    r = subprocess.run([sys.executable, "-c", _CHILD, ROOT], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ))
    assert r.returncode == 0 and "child ok" in r.stdout, r.stdout + r.stderr


def test_noalloc_rejects_problems_beyond_its_scratch():
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    dummy = C.c_void_p(256)
    # B*K above 4,194,304 activations, and B above 4096 rows
    for B, K in ((1024, 8192), (4097, 16), (1025, 4096)):
        st = lib.dgx_gemm_w8a8_noalloc(dummy, dummy, dummy, None, dummy, B, 64, K, None)
        assert st == _lib.DGX_EINVAL
        assert b"exceeds the fixed scratch" in lib.dgx_last_error()
