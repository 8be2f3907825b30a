"""GPU: failure detection on one GPU, without a device fault. A bounded
device wait that nothing completes must end with DGX_ETIMEOUT from
dgx_sync_check and leave the context usable; an injected host-side fault
must surface as an error and leave the next calls working.

The waits are the library's own: the cross-rank completion wait of the
column-parallel GEMM (its flag never raised, budget 2 ms) and the mbarrier
wait of the tensor-core pipelines (a barrier that never completes, its fixed
budget of about one second)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _probe(kind, flag, expect, timeout_us):
    from dreamcompiler_b200 import _lib
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("dgx_wait_probe", kind, flag.data_ptr() if flag is not None else None, expect, timeout_us, s)
    return _lib.load().dgx_sync_check(s)


def _gemm_still_works(dgx):
    A = torch.randn(256, 128, device="cuda").bfloat16()
    B = torch.randn(128, 192, device="cuda").bfloat16()
    C = dgx.gemm(A, B)
    dgx.sync_check()
    ref = A.double() @ B.double()
    assert ((C.double() - ref).abs().max() / ref.abs().max()).item() < 1e-2


def test_flag_wait_times_out_and_the_context_survives(dgx):
    from dreamcompiler_b200 import _lib
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert _probe(0, flag, 1, 2000) == _lib.DGX_ETIMEOUT
    assert b"1=wait timeout" in _lib.load().dgx_last_error()
    # the error word was cleared by the check; the device still computes
    assert _lib.load().dgx_sync_check(torch.cuda.current_stream().cuda_stream) == _lib.DGX_OK
    _gemm_still_works(dgx)
    flag.fill_(5)
    assert _probe(0, flag, 5, 2000) == _lib.DGX_OK


def test_mbarrier_wait_times_out_and_the_context_survives(dgx):
    from dreamcompiler_b200 import _lib
    assert _probe(1, None, 0, 0) == _lib.DGX_OK           # completed barrier: no timeout
    assert _probe(1, None, 1, 0) == _lib.DGX_ETIMEOUT     # never completed: ~1 s, then the error word
    _gemm_still_works(dgx)


def test_injected_fault_surfaces_and_clears(dgx):
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    q, k, v = (torch.randn(2, 256, 64, device="cuda").bfloat16() for _ in range(3))
    try:
        assert lib.dgx_fault_inject(2, _lib.DGX_ETIMEOUT) == _lib.DGX_OK
        O1, _ = dgx.flash_fwd(q, k, v)
        with pytest.raises(_lib.DgxError) as e:
            dgx.flash_fwd(q, k, v)
        assert "injected fault at call 2 (dgx_flash_fwd)" in str(e.value)
        O3, _ = dgx.flash_fwd(q, k, v)
        dgx.sync_check()
        assert torch.equal(O1, O3)
    finally:
        lib.dgx_fault_inject(0, 0)
    _gemm_still_works(dgx)
