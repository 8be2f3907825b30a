"""TEST INFRASTRUCTURE: ctypes binding of the reference Dream runtime.

oracle/_ref/libdream_ref.so is the reference runtime (heellowdsf/
DreamCompiler runtime/) compiled from its own sources by build_ref.sh. This
module drives it through its public C ABI exactly as a libdream C program
would (interop/dream.h): every op takes and returns ``Tensor*``; the first
fields of ``struct Tensor`` (runtime/runtime.h:49-54: double* data, double*
grad, int size, int d0..d3) are read directly, as compiled Dream code does.

Used to generate golden vectors (tests/golden/make_golden.py), to pin the
oracle, and as the timed reference CPU path in bench.py. No torch import, so
spawned worker processes start quickly.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libdream_ref.so")


class TensorHead(C.Structure):
    # runtime/runtime.h:49-54 — the LLVM-visible prefix of struct Tensor.
    _fields_ = [("data", C.POINTER(C.c_double)), ("grad", C.POINTER(C.c_double)), ("size", C.c_int),
                ("d0", C.c_int), ("d1", C.c_int), ("d2", C.c_int), ("d3", C.c_int)]


TP = C.POINTER(TensorHead)
_lib = None

_SIG = {
    "create_scalar": [C.c_double],
    "alloc_tensor": [C.c_int, C.c_int, C.c_int, C.c_int],
    "dream_set_seed": [TP],
    "dream_randn": [TP, TP],
    "tensor_matmul": [TP, TP],
    "tensor_mul": [TP, TP],
    "sum": [TP],
    "backward": [TP],
    "dream_set_precision": [TP, C.c_int],
    "dream_flash_attention": [TP, TP, TP, TP, TP, TP, TP],
    "dream_attention_causal": [TP, TP, TP, TP, TP, TP],
    "dream_attention": [TP, TP, TP, TP, TP, TP],
    "dream_tp_matmul_column": [TP, TP, TP],
    "dream_linear": [TP, TP, TP],
    "dream_linear_relu": [TP, TP, TP],
    "dream_bmm": [TP, TP, TP, TP, TP, TP],
    "tensor_decref": [TP],
    "tensor_add": [TP, TP],
    "dream_reshape_nd": [TP, TP, TP],
    "dream_embedding": [TP, TP],
    "dream_layer_norm": [TP],
    "dream_gelu": [TP],
    "dream_log_softmax": [TP],
    "dream_nll_loss": [TP, TP],
    "dream_adamw_update": [TP, TP, TP, TP, TP, TP],
    "zero_grad": [TP],
    "dream_str_create": [C.c_char_p],
    "dream_conv2d": [TP] * 7,
    "dream_conv2d_padded": [TP] * 9,
    "dream_ckpt_new": [],
    "dream_ckpt_add": [TP, TP, TP],
    "dream_export_c_header_int8": [TP, TP, TP],
    "gemm_selftest": [],
    "flash_attention_selftest": [],
    "tensor_parallel_selftest": [],
}


def available() -> bool:
    return os.path.exists(LIB)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB} not built (oracle/build_ref.sh needs the reference sources)")
        _lib = C.CDLL(LIB)
        for name, args in _SIG.items():
            f = getattr(_lib, name)
            f.argtypes = args
            f.restype = TP
    return _lib


def scalar(v: float):
    return lib().create_scalar(float(v))


def set_seed(seed: int) -> None:
    lib().dream_set_seed(scalar(seed))


def randn(rows: int, cols: int):
    return lib().dream_randn(scalar(rows), scalar(cols))


def tensor(a: np.ndarray):
    """New reference tensor (rows x cols, f64) holding a copy of `a`."""
    a = np.ascontiguousarray(a, dtype=np.float64)
    rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.size)
    t = lib().alloc_tensor(rows, cols, 1, 1)
    C.memmove(t.contents.data, a.ctypes.data, a.nbytes)
    return t


def data(t, shape=None) -> np.ndarray:
    h = t.contents
    out = np.ctypeslib.as_array(h.data, shape=(h.size,)).copy()
    return out.reshape(shape if shape is not None else (h.d0, h.d1))


def grad(t, shape=None) -> np.ndarray:
    h = t.contents
    out = np.ctypeslib.as_array(h.grad, shape=(h.size,)).copy()
    return out.reshape(shape if shape is not None else (h.d0, h.d1))


def call(name: str, *args):
    return getattr(lib(), name)(*args)
