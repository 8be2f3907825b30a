"""CPU: host-side fault injection (dgx_fault_inject / DGX_FAIL_AT). The n-th
call to an entry point that launches device work returns the chosen error
status and launches nothing, so the failure paths above the library (the
Dream op mirror's RUNTIME ERROR, a rank that leaves between steps) can be
tested without faulting a GPU. These calls fail or succeed before any device
work, so they run without a GPU."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT


@pytest.fixture()
def lib():
    from dreamcompiler_b200 import _lib
    lib = _lib.load()
    yield lib
    assert lib.dgx_fault_inject(0, 0) == _lib.DGX_OK


def _gemm_empty(lib):
    from dreamcompiler_b200 import _lib
    # M = 0: a valid call that does no device work
    return lib.dgx_gemm(None, None, None, 0, 4, 4, 4, 4, 4, 0, 0, _lib.DGX_BF16, _lib.DGX_F32, 0, None, 0, 0.0,
                        None, 0, None)


def test_nth_call_fails_with_the_chosen_status(lib):
    from dreamcompiler_b200 import _lib
    assert lib.dgx_fault_inject(3, _lib.DGX_ENCCL) == _lib.DGX_OK
    got = [_gemm_empty(lib) for _ in range(5)]
    assert got == [_lib.DGX_OK, _lib.DGX_OK, _lib.DGX_ENCCL, _lib.DGX_OK, _lib.DGX_OK]
    assert lib.dgx_fault_calls() == 5
    # the message names the call and the entry point
    assert lib.dgx_fault_inject(1, _lib.DGX_ETIMEOUT) == _lib.DGX_OK
    assert _gemm_empty(lib) == _lib.DGX_ETIMEOUT
    assert lib.dgx_last_error() == b"injected fault at call 1 (dgx_gemm)"


def test_python_wrapper_raises_on_an_injected_fault(lib):
    from dreamcompiler_b200 import _lib
    assert lib.dgx_fault_inject(1, _lib.DGX_ETIMEOUT) == _lib.DGX_OK
    with pytest.raises(_lib.DgxError) as e:
        _lib.call("dgx_flash_fwd", None, None, None, None, None, 0, 128, 64, 0.125, 1, _lib.DGX_BF16, None)
    assert e.value.status == _lib.DGX_ETIMEOUT and "injected fault" in str(e.value)


def test_off_and_invalid_settings(lib):
    from dreamcompiler_b200 import _lib
    assert lib.dgx_fault_inject(0, 0) == _lib.DGX_OK
    assert all(_gemm_empty(lib) == _lib.DGX_OK for _ in range(4))
    assert lib.dgx_fault_inject(2, _lib.DGX_OK) == _lib.DGX_EINVAL      # not an error status
    assert lib.dgx_fault_inject(-1, _lib.DGX_ETIMEOUT) == _lib.DGX_EINVAL


_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1])
from dreamcompiler_b200 import _lib
lib = _lib.load()
args = (None, None, None, 0, 4, 4, 4, 4, 4, 0, 0, _lib.DGX_BF16, _lib.DGX_F32, 0, None, 0, 0.0, None, 0, None)
print(",".join(str(lib.dgx_gemm(*args)) for _ in range(3)))
"""


@pytest.mark.parametrize("env,want", [("2", "0,4,0"), ("1:3", "3,0,0"), ("0", "0,0,0"), ("3:99", "0,0,4")])
def test_environment_setting(env, want):
    r = subprocess.run([sys.executable, "-c", _CHILD, ROOT], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, DGX_FAIL_AT=env))
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == want
