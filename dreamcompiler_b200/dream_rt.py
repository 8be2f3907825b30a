"""ctypes binding of libdream_b200.so (include/dream_b200.h): the Dream
runtime's op names over the B200 kernels. Mirrors oracle/refrt.py, the
binding of the reference runtime, so a test can run the same Dream-level
program on both and compare."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libdream_b200.so")


class TensorHead(C.Structure):
    # the LLVM-visible prefix of struct Tensor (runtime/runtime.h:49-54)
    _fields_ = [("data", C.POINTER(C.c_double)), ("grad", C.POINTER(C.c_double)), ("size", C.c_int),
                ("d0", C.c_int), ("d1", C.c_int), ("d2", C.c_int), ("d3", C.c_int)]


TP = C.POINTER(TensorHead)
_SIG = {
    "alloc_tensor": [C.c_int] * 4, "create_scalar": [C.c_double], "tensor_incref": [TP], "tensor_decref": [TP],
    "tensor_get_grad": [TP], "zero_grad": [TP], "dream_set_seed": [TP], "dream_randn": [TP, TP],
    "dream_set_precision": [TP, C.c_int], "dream_enable_fp16": [], "tensor_matmul": [TP, TP],
    "dream_linear": [TP, TP, TP], "dream_linear_relu": [TP, TP, TP], "dream_bmm": [TP] * 6,
    "dream_flash_attention": [TP] * 7, "dream_conv2d": [TP] * 7, "dream_conv2d_padded": [TP] * 9, "dream_attention": [TP] * 6, "dream_attention_causal": [TP] * 6, "dream_tp_matmul_column": [TP] * 3, "tensor_mul": [TP, TP], "sum": [TP],
    "backward": [TP],
}
_rt = None


def load() -> C.CDLL:
    global _rt
    if _rt is None:
        _lib.load()  # libdgx first (RTLD_GLOBAL)
        if not os.path.exists(LIB):
            raise ImportError(f"{LIB} not built; run python -m dreamcompiler_b200.build")
        _rt = C.CDLL(LIB)
        for name, args in _SIG.items():
            f = getattr(_rt, name)
            f.argtypes = args
            f.restype = TP
    return _rt


def scalar(v: float):
    return load().create_scalar(float(v))


def tensor(a: np.ndarray):
    a = np.ascontiguousarray(a, dtype=np.float64)
    rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.size)
    t = load().alloc_tensor(rows, cols, 1, 1)
    C.memmove(t.contents.data, a.ctypes.data, a.nbytes)
    return t


def data(t, shape=None) -> np.ndarray:
    h = t.contents
    return np.ctypeslib.as_array(h.data, shape=(h.size,)).copy().reshape(shape or (h.d0, h.d1))


def grad(t, shape=None) -> np.ndarray:
    h = t.contents
    return np.ctypeslib.as_array(h.grad, shape=(h.size,)).copy().reshape(shape or (h.d0, h.d1))


def call(name: str, *args):
    return getattr(load(), name)(*args)
