"""CPU: the C-ABI libraries load, export every symbol include/*.h declares,
and reject bad arguments before touching the device."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT

INCLUDE = os.path.join(ROOT, "include")


def declared(header: str):
    text = open(os.path.join(INCLUDE, header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:dgx|dream|tensor)_\w+|backward)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from dreamcompiler_b200 import _lib
    return _lib.load()


def test_libdgx_exports_every_declared_symbol(lib):
    names = declared("dgx.h")
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"libdgx.so does not export {n}"


def test_python_binding_covers_header():
    from dreamcompiler_b200 import _lib
    assert set(declared("dgx.h")) <= set(_lib.SIGNATURES)


def test_python_binding_arity_matches_header():
    """Every ctypes signature has as many parameters as its prototype."""
    from dreamcompiler_b200 import _lib
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(INCLUDE, "dgx.h")).read(), flags=re.S)
    protos = dict(re.findall(r"\b(dgx_\w+)\s*\(([^)]*)\)\s*;", text))
    assert len(protos) >= 15
    for name, params in protos.items():
        n = 0 if params.strip() in ("", "void") else params.count(",") + 1
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: binding has {len(_lib.SIGNATURES[name][1])}, header {n}"


def test_dream_runtime_exports(lib):
    from dreamcompiler_b200 import dream_rt
    rt = dream_rt.load()
    for n in declared("dream_b200.h"):
        assert hasattr(rt, n), f"libdream_b200.so does not export {n}"


def test_version_and_last_error(lib):
    assert b"sm_100a" in lib.dgx_version()
    from dreamcompiler_b200 import _lib
    st = lib.dgx_gemm(None, None, None, -1, 4, 4, 4, 4, 4, 0, 0, _lib.DGX_BF16, _lib.DGX_F32, 0, None, 0, 0.0,
                      None, 0, None)
    assert st == _lib.DGX_EINVAL
    assert b"negative" in lib.dgx_last_error()


def test_argument_validation_without_device(lib):
    from dreamcompiler_b200 import _lib as L
    # empty problems are a no-op
    assert lib.dgx_gemm(None, None, None, 0, 5, 5, 5, 5, 5, 0, 0, L.DGX_BF16, L.DGX_F32, 0, None, 0, 0.0, None, 0,
                        None) == L.DGX_OK
    # null operands, bad enums, bias epilogue without bias, short leading dims
    assert lib.dgx_gemm(None, None, None, 4, 4, 4, 4, 4, 4, 0, 0, L.DGX_BF16, L.DGX_F32, 0, None, 0, 0.0, None, 0,
                        None) == L.DGX_EINVAL
    fake = C.c_void_p(16)
    assert lib.dgx_gemm(fake, fake, fake, 4, 4, 4, 4, 4, 4, 0, 0, 7, L.DGX_F32, 0, None, 0, 0.0, None, 0,
                        None) == L.DGX_EINVAL
    assert lib.dgx_gemm(fake, fake, fake, 4, 4, 4, 4, 4, 4, 0, 0, L.DGX_BF16, L.DGX_F32, 0, None, L.DGX_EPI_BIAS,
                        0.0, None, 0, None) == L.DGX_EINVAL
    assert lib.dgx_gemm(fake, fake, fake, 4, 4, 8, 2, 4, 4, 0, 0, L.DGX_BF16, L.DGX_F32, 0, None, 0, 0.0, None, 0,
                        None) == L.DGX_EINVAL
    assert lib.dgx_flash_fwd(fake, fake, fake, fake, None, 1, 16, 64, 0.125, 1, L.DGX_F32, None) == L.DGX_EUNSUPPORTED
    assert lib.dgx_flash_fwd(None, None, None, None, None, 1, 16, 64, 0.125, 1, L.DGX_BF16, None) == L.DGX_EINVAL
    assert lib.dgx_flash_fwd(fake, fake, fake, fake, None, 1, 16, 0, 0.125, 1, L.DGX_BF16, None) == L.DGX_EINVAL
    assert lib.dgx_gemm_w8(fake, fake, fake, None, fake, 1, 4, 4, 5, None) == L.DGX_EINVAL
    assert lib.dgx_gemm_i8i32(None, None, None, 2, 2, 2, None) == L.DGX_EINVAL


def test_workspace_sizes(lib):
    from dreamcompiler_b200 import _lib as L
    # 3xTF32 keeps hi+lo planes of both operands, K padded to 4
    assert lib.dgx_gemm_workspace_size(1024, 512, 1023, 0, 0, L.DGX_F32, L.DGX_F32_3XTF32) == \
        2 * (1024 * 1024 + 512 * 1024) * 4
    assert lib.dgx_gemm_workspace_size(64, 64, 64, 0, 0, L.DGX_BF16, 0) == 0
    assert lib.dgx_gemm_workspace_size(64, 64, 64, 0, 0, L.DGX_F32, L.DGX_F32_FFMA) == 0
    # flash backward: fp32 dQ accumulator + 2 padded row-statistic vectors
    assert lib.dgx_flash_bwd_workspace_size(8, 300, 64) == (8 * 300 * 64 + 2 * 8 * 384) * 4


@pytest.mark.parametrize("N", [1, 7, 24, 23, 4096, 16384, 16385])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 5, 7, 8])
def test_tp_shard_matches_reference_widths(lib, orc, N, G):
    c0, nc = C.c_int(), C.c_int()
    for g in range(G):
        lib.dgx_tp_shard(N, G, g, C.byref(c0), C.byref(nc))
        assert (c0.value, nc.value) == orc.tp_shard(N, G, g)


def test_reference_runtime_with_b200_backend_loads():
    """The reference runtime built with the B200 backend (refside/build.sh)
    exports the reference's ops and the backend's op counter."""
    from dreamcompiler_b200 import refside
    if not refside.available():
        pytest.skip("libdream_ref_b200.so needs the reference sources to build")
    rt = refside.load()
    for n in ("tensor_matmul", "dream_linear", "dream_linear_relu", "dream_flash_attention", "backward",
              "dream_tp_matmul_column", "dream_set_precision", "dream_b200_count"):
        assert hasattr(rt, n)
    assert rt.dream_b200_count(0) == 0 and rt.dream_b200_count(99) == -1
