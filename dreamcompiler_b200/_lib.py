"""ctypes binding of libdgx (include/dgx.h).

Every call goes through the C ABI exactly as a C or cgo caller would bind it;
this module only converts Python arguments to pointers and sizes and turns a
non-OK status into a ``DgxError``. There is no fallback: if the shared
library is missing the import of a compute entry point fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdgx.so")

DGX_OK, DGX_EINVAL, DGX_ECUDA, DGX_ENCCL, DGX_ETIMEOUT, DGX_EUNSUPPORTED, DGX_ENOMEM = range(7)
DGX_F32, DGX_BF16, DGX_I8, DGX_F64 = 0, 1, 2, 3
DGX_EPI_NONE, DGX_EPI_BIAS, DGX_EPI_BIAS_RELU, DGX_EPI_RELU = 0, 1, 2, 3
DGX_F32_3XTF32, DGX_F32_FFMA = 0, 1

STATUS_NAMES = {0: "DGX_OK", 1: "DGX_EINVAL", 2: "DGX_ECUDA", 3: "DGX_ENCCL", 4: "DGX_ETIMEOUT",
                5: "DGX_EUNSUPPORTED", 6: "DGX_ENOMEM"}


class DgxError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes). Must list every function include/dgx.h declares.
SIGNATURES = {
    "dgx_version": (C.c_char_p, []),
    "dgx_last_error": (C.c_char_p, []),
    "dgx_init": (_i, [_i]),
    "dgx_sync_check": (_i, [_vp]),
    "dgx_set_timer_events": (None, [_vp, _vp]),
    "dgx_stream_create": (_i, [_vp]),
    "dgx_device_alloc": (_i, [_sz, _vp]),
    "dgx_device_free": (_i, [_vp]),
    "dgx_copy": (_i, [_vp, _vp, _sz, _i, _vp]),
    "dgx_fault_inject": (_i, [C.c_longlong, _i]),
    "dgx_fault_calls": (C.c_longlong, []),
    "dgx_wait_probe": (_i, [_i, _vp, C.c_ulonglong, _i, _vp]),
    "dgx_convert": (_i, [_vp, _i, _vp, _i, _sz, _i, _vp]),
    "dgx_fingerprint": (_i, [_vp, _sz, _vp, _vp]),
    "dgx_gemm": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _f, _vp, _sz, _vp]),
    "dgx_gemm_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "dgx_gemm_f64": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _i, C.c_double, _vp]),
    "dgx_gemm_set_algo": (_i, [_i]),
    "dgx_bmm": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "dgx_conv2d_fwd": (_i, [_vp] * 4 + [_i] * 10 + [_vp]),
    "dgx_conv2d_bwd": (_i, [_vp] * 5 + [_i] * 11 + [_vp]),
    "dgx_conv2d_workspace_size": (_sz, [_i] * 10),
    "dgx_flash_fwd_rows": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _f, _i, _vp]),
    "dgx_flash_bwd_rows": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _vp, _i, _vp, _i, _vp, _i,
                                _i, _i, _i, _i, _f, _i, _vp, _sz, _vp]),
    "dgx_dense_q": (_i, [_vp, _vp, _f, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "dgx_gemm_batched": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, C.c_longlong, C.c_longlong, C.c_longlong,
                               _i, _i, _i, _i, _f, _vp]),
    "dgx_flash_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp]),
    "dgx_flash_bwd": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp]),
    "dgx_flash_bwd_workspace_size": (_sz, [_i, _i, _i]),
    "dgx_flash_set_deterministic": (_i, [_i]),
    "dgx_gemm_w8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "dgx_gemm_w8a8_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "dgx_gemm_i8i32": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "dgx_quantize_rows_i8": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "dgx_layernorm_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "dgx_layernorm_bwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "dgx_layernorm_bwd_x16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "dgx_gelu_fwd": (_i, [_vp, _i, _vp, C.c_longlong, _vp]),
    "dgx_gelu_bwd": (_i, [_vp, _i, _vp, _i, _vp, C.c_longlong, _vp]),
    "dgx_embedding_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "dgx_embedding_bwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "dgx_softmax_nll": (_i, [_vp, _i, _i, _vp, _i, _vp, _vp, _i, _vp]),
    "dgx_adamw": (_i, [_vp, _vp, _vp, _vp, C.c_longlong, _f, _f, _f, _f, _f, _i, _vp, _vp]),
    "dgx_colsum": (_i, [_vp, _i, _vp, _i, _i, _i, _vp]),
    "dgx_rows_to_heads": (_i, [_vp, _i, _i, _i, _vp, _i, _i, _i, _i, _vp]),
    "dgx_heads_to_rows": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "dgx_tp_shard": (None, [_i, _i, _i, C.POINTER(_i), C.POINTER(_i)]),
    "dgx_tp_export": (_i, [_vp, _sz, _vp, _sz]),
    "dgx_tp_handle_size": (_sz, []),
    "dgx_tp_open": (_i, [_i, _i, _vp]),
    "dgx_tp_gemm_colsplit": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "dgx_tp_close": (_i, []),
}

_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libdgx.so (built by dreamcompiler_b200.build) and bind signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"libdgx.so not built at {path}; run python -m dreamcompiler_b200.build")
    lib = C.CDLL(path, mode=C.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, where: str) -> None:
    if status != DGX_OK:
        msg = load().dgx_last_error().decode(errors="replace")
        raise DgxError(status, where, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
