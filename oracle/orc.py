"""TEST INFRASTRUCTURE: numpy-facing binding of liboracle.so (dream_oracle.cpp).

``build()`` compiles the library with g++ (OpenMP) next to this file; every
wrapper takes/returns numpy arrays and calls the C restatement.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "dream_oracle.cpp")
SRC_RNG = os.path.join(HERE, "dream_oracle_rng.cpp")
# The RNG translation unit uses the reference runtime's compile flags so the
# normal_distribution stream matches it bit for bit (see dream_oracle_rng.cpp).
RNG_FLAGS = ["-O3", "-ffast-math", "-mavx2", "-mfma", "-fno-math-errno"]
LIB = os.path.join(HERE, "liboracle.so")

_lib = None


def build(force: bool = False) -> str:
    newest = max(os.path.getmtime(SRC), os.path.getmtime(SRC_RNG), os.path.getmtime(__file__))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        rng_obj = LIB + ".rng.o"
        subprocess.run(["g++", "-std=c++17", "-fPIC", "-c", SRC_RNG, "-o", rng_obj] + RNG_FLAGS, check=True)
        subprocess.run(["g++", "-O2", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-Wall", SRC, rng_obj,
                        "-o", LIB], check=True)
        os.remove(rng_obj)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB)
        _lib.orc_to_bf16.restype = C.c_float
        _lib.orc_to_bf16.argtypes = [C.c_float]
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- RNG
def set_seed(seed: int) -> None:
    lib().orc_set_seed(C.c_uint(seed))


def randn(*shape) -> np.ndarray:
    out = np.empty(shape, dtype=np.float64)
    lib().orc_randn(_p(out), C.c_long(out.size))
    return out


def rand_uniform(shape, lo: float, hi: float) -> np.ndarray:
    out = np.empty(shape, dtype=np.float64)
    lib().orc_rand_uniform(_p(out), C.c_long(out.size), C.c_double(lo), C.c_double(hi))
    return out


# ---------------------------------------------------------------- bf16
def round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_round_bf16(_p(x), _p(out), C.c_long(x.size))
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_bf16_bits(_p(x), _p(out), C.c_long(x.size))
    return out


# ---------------------------------------------------------------- GEMM
def gemm_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    M, K = A.shape
    N = B.shape[1]
    C_ = np.empty((M, N), np.float64)
    lib().orc_gemm_f64(_p(A), _p(B), _p(C_), M, K, N)
    return C_


def gemm_rows_f64(A: np.ndarray, B: np.ndarray, rows: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    rows = np.ascontiguousarray(rows, np.int32)
    K, N = B.shape
    C_ = np.empty((rows.size, N), np.float64)
    lib().orc_gemm_rows_f64(_p(A), _p(B), _p(C_), _p(rows), rows.size, K, N)
    return C_


def gemm_f32(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    C_ = np.empty((M, N), np.float32)
    lib().orc_gemm_f32(_p(A), _p(B), _p(C_), M, K, N)
    return C_


def matmul_bwd(A, B, dY, dA=None, dB=None):
    A, B, dY = (np.ascontiguousarray(t, np.float64) for t in (A, B, dY))
    M, K = A.shape
    N = B.shape[1]
    dA = np.zeros((M, K)) if dA is None else dA
    dB = np.zeros((K, N)) if dB is None else dB
    lib().orc_matmul_bwd(_p(A), _p(B), _p(dY), _p(dA), _p(dB), M, K, N)
    return dA, dB


def bmm(A, B):
    """A [batch, M, K], B [batch, K, N] float64 -> C [batch, M, N] (dream_bmm)."""
    A, B = (np.ascontiguousarray(t, np.float64) for t in (A, B))
    nb, M, K = A.shape
    N = B.shape[2]
    C_ = np.empty((nb, M, N))
    lib().orc_bmm_f64(_p(A), _p(B), _p(C_), nb, M, K, N)
    return C_


def bmm_bwd(A, B, dC):
    A, B, dC = (np.ascontiguousarray(t, np.float64) for t in (A, B, dC))
    nb, M, K = A.shape
    N = B.shape[2]
    dA, dB = np.zeros_like(A), np.zeros_like(B)
    lib().orc_bmm_bwd(_p(A), _p(B), _p(dC), _p(dA), _p(dB), nb, M, K, N)
    return dA, dB


def linear(X, W, b, relu=False):
    X, W = (np.ascontiguousarray(t, np.float64) for t in (X, W))
    b = None if b is None else np.ascontiguousarray(b, np.float64)
    N, din = X.shape
    dout = W.shape[0]
    Y = np.empty((N, dout))
    lib().orc_linear(_p(X), _p(W), None if b is None else _p(b), _p(Y), N, din, dout, int(relu))
    return Y


def linear_bwd(X, W, Y, dY, relu=False):
    X, W, Y, dY = (np.ascontiguousarray(t, np.float64) for t in (X, W, Y, dY))
    N, din = X.shape
    dout = W.shape[0]
    dX, dW, db = np.zeros((N, din)), np.zeros((dout, din)), np.zeros(dout)
    lib().orc_linear_bwd(_p(X), _p(W), _p(Y), _p(dY), _p(dX), _p(dW), _p(db), N, din, dout, int(relu))
    return dX, dW, db


# ---------------------------------------------------------------- attention
def flash_fwd(Q, K, V, block: int = 64):
    """Q, K, V: [B, S, dk] float64. Returns (O, LSE[B, S] natural log)."""
    Q, K, V = (np.ascontiguousarray(t, np.float64) for t in (Q, K, V))
    B, S, dk = Q.shape
    O = np.empty_like(Q)
    lse = np.empty((B, S))
    lib().orc_flash_fwd(_p(Q), _p(K), _p(V), _p(O), _p(lse), B, S, dk, block)
    return O, lse


def flash_bwd(Q, K, V, dO):
    Q, K, V, dO = (np.ascontiguousarray(t, np.float64) for t in (Q, K, V, dO))
    B, S, dk = Q.shape
    dQ, dK, dV = np.zeros_like(Q), np.zeros_like(K), np.zeros_like(V)
    lib().orc_flash_bwd(_p(Q), _p(K), _p(V), _p(dO), _p(dQ), _p(dK), _p(dV), B, S, dk)
    return dQ, dK, dV


def attention(Q, K, V, causal=True):
    Q, K, V = (np.ascontiguousarray(t, np.float64) for t in (Q, K, V))
    B, S, dk = Q.shape
    O = np.empty_like(Q)
    lib().orc_attention(_p(Q), _p(K), _p(V), _p(O), B, S, dk, int(causal))
    return O


def attention_bwd(Q, K, V, dO, causal=True):
    Q, K, V, dO = (np.ascontiguousarray(t, np.float64) for t in (Q, K, V, dO))
    B, S, dk = Q.shape
    dQ, dK, dV = np.zeros_like(Q), np.zeros_like(K), np.zeros_like(V)
    lib().orc_attention_bwd(_p(Q), _p(K), _p(V), _p(dO), _p(dQ), _p(dK), _p(dV), B, S, dk, int(causal))
    return dQ, dK, dV


# ---------------------------------------------------------------- convolution
def conv_out(H, W, KH, KW, pad=0, stride=1):
    return (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1


def conv2d_fwd(X, K, bias, KH, KW, pad=0, stride=1):
    """X [N, Cin, H, W], K [Cout, Cin*KH*KW], bias [Cout] or None -> Y [N, Cout, OH, OW] (f64)."""
    X, K = (np.ascontiguousarray(t, np.float64) for t in (X, K))
    N, Cin, H, W = X.shape
    Cout = K.shape[0]
    OH, OW = conv_out(H, W, KH, KW, pad, stride)
    Y = np.empty((N, Cout, OH, OW))
    bp = None if bias is None else _p(np.ascontiguousarray(bias, np.float64))
    lib().orc_conv2d_fwd(_p(X), _p(K), bp, _p(Y), N, Cin, H, W, Cout, KH, KW, pad, stride)
    return Y


def conv2d_bwd(X, K, dY, KH, KW, pad=0, stride=1):
    X, K, dY = (np.ascontiguousarray(t, np.float64) for t in (X, K, dY))
    N, Cin, H, W = X.shape
    Cout = K.shape[0]
    dX, dK = np.zeros_like(X), np.zeros_like(K)
    lib().orc_conv2d_bwd(_p(X), _p(K), _p(dY), _p(dX), _p(dK), N, Cin, H, W, Cout, KH, KW, pad, stride)
    return dX, dK


# ---------------------------------------------------------------- int8
def quantize_per_tensor(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float64)
    q = np.empty(w.shape, np.int8)
    s = C.c_double(0)
    lib().orc_quantize_per_tensor(_p(w), C.c_long(w.size), _p(q), C.byref(s))
    return q, s.value


def dense_q(X, W, scale, bias):
    X = np.ascontiguousarray(X, np.float32)
    W = np.ascontiguousarray(W, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    B, K = X.shape
    N = W.shape[0]
    Y = np.empty((B, N), np.float32)
    bp = None if bias is None else _p(np.ascontiguousarray(bias, np.float32))
    lib().orc_dense_q(_p(X), _p(W), _p(scale), bp, _p(Y), B, N, K)
    return Y


def i8_gemm(Xq, W):
    Xq = np.ascontiguousarray(Xq, np.int8)
    W = np.ascontiguousarray(W, np.int8)
    B, K = Xq.shape
    N = W.shape[0]
    acc = np.empty((B, N), np.int32)
    lib().orc_i8_gemm(_p(Xq), _p(W), _p(acc), B, N, K)
    return acc


def quantize_rows(X):
    X = np.ascontiguousarray(X, np.float32)
    B, K = X.shape
    Xq = np.empty((B, K), np.int8)
    sx = np.empty(B, np.float32)
    lib().orc_quantize_rows(_p(X), _p(Xq), _p(sx), B, K)
    return Xq, sx


# ---------------------------------------------------------------- tensor parallel
def tp_shard(N: int, G: int, g: int):
    c0, nc = C.c_int(0), C.c_int(0)
    lib().orc_tp_shard(N, G, g, C.byref(c0), C.byref(nc))
    return c0.value, nc.value


def tp_matmul_column(X, W, G):
    X, W = (np.ascontiguousarray(t, np.float64) for t in (X, W))
    M, K = X.shape
    N = W.shape[1]
    Y = np.empty((M, N))
    lib().orc_tp_matmul_column(_p(X), _p(W), _p(Y), M, K, N, G)
    return Y
