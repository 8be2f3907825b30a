"""ctypes binding of libdream_ref_b200.so: the reference Dream runtime
(heellowdsf/DreamCompiler runtime/) built with this package's B200 backend
(b200.inc, build.sh). It exports the reference's own extern "C" ops on the
reference's own struct Tensor; tensor_matmul, dream_linear,
dream_flash_attention and their backward branches run on the B200 through
libdgx, everything else is the reference's code.

A C program or a compiled Dream program links this library in place of the
reference's libdream; Python drives it the same way here (tests, bench).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .. import _lib

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libdream_ref_b200.so")

# dream_b200_count(i): device runs of each hooked op, then operand uploads and
# device-copy reuses (b200.inc, enum b200::Op).
COUNTS = ["matmul_f64", "matmul_f32", "matmul_bf16", "linear", "flash_fwd", "matmul_bwd", "linear_bwd",
          "flash_bwd", "uploads", "mirror_hits"]


class TensorHead(C.Structure):
    # the LLVM-visible prefix of struct Tensor (runtime/runtime.h:49-54)
    _fields_ = [("data", C.POINTER(C.c_double)), ("grad", C.POINTER(C.c_double)), ("size", C.c_int),
                ("d0", C.c_int), ("d1", C.c_int), ("d2", C.c_int), ("d3", C.c_int)]


TP = C.POINTER(TensorHead)
_SIG = {
    "create_scalar": [C.c_double], "alloc_tensor": [C.c_int] * 4, "tensor_decref": [TP],
    "dream_set_seed": [TP], "dream_randn": [TP, TP], "tensor_matmul": [TP, TP], "tensor_mul": [TP, TP],
    "sum": [TP], "backward": [TP], "zero_grad": [TP], "dream_set_precision": [TP, C.c_int],
    "dream_enable_fp16": [], "dream_linear": [TP] * 3, "dream_linear_relu": [TP] * 3,
    "dream_flash_attention": [TP] * 7, "dream_tp_matmul_column": [TP] * 3,
    "tensor_parallel_selftest": [], "flash_attention_selftest": [],
}
_rt = None


def available() -> bool:
    return os.path.exists(LIB)


def load() -> C.CDLL:
    global _rt
    if _rt is None:
        _lib.load()  # libdgx first
        if not available():
            raise ImportError(f"{LIB} not built; run dreamcompiler_b200/refside/build.sh <DreamCompiler checkout>")
        _rt = C.CDLL(LIB)
        for name, args in _SIG.items():
            f = getattr(_rt, name)
            f.argtypes = args
            f.restype = TP
        _rt.dream_b200_count.argtypes = [C.c_int]
        _rt.dream_b200_count.restype = C.c_longlong
        _rt.dream_b200_time_us.argtypes = [C.c_int]
        _rt.dream_b200_time_us.restype = C.c_double
    return _rt


def counts() -> dict:
    rt = load()
    return {name: rt.dream_b200_count(i) for i, name in enumerate(COUNTS)}


TIMES = ["fingerprint", "upload", "download", "ops"]


def times_us() -> dict:
    """Host wall time the backend spent so far, by kind (microseconds)."""
    rt = load()
    return {name: rt.dream_b200_time_us(i) for i, name in enumerate(TIMES)}


def scalar(v: float):
    return load().create_scalar(float(v))


def tensor(a: np.ndarray):
    """New runtime tensor (rows x cols, f64) holding a copy of `a`."""
    a = np.ascontiguousarray(a, dtype=np.float64)
    rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.size)
    t = load().alloc_tensor(rows, cols, 1, 1)
    C.memmove(t.contents.data, a.ctypes.data, a.nbytes)
    return t


def view(t, field: str = "data") -> np.ndarray:
    """The tensor's host buffer (no copy): writes go to the runtime's memory."""
    h = t.contents
    return np.ctypeslib.as_array(getattr(h, field), shape=(h.size,))


def data(t, shape=None) -> np.ndarray:
    h = t.contents
    return view(t).copy().reshape(shape if shape is not None else (h.d0, h.d1))


def grad(t, shape=None) -> np.ndarray:
    h = t.contents
    return view(t, "grad").copy().reshape(shape if shape is not None else (h.d0, h.d1))


def call(name: str, *args):
    return getattr(load(), name)(*args)
