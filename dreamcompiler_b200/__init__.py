"""dreamcompiler_b200 — B200-native hot path of the Dream tensor runtime.

The product is two native libraries built from this package:

* ``libdgx.so`` — hand-written sm_100a kernels (tcgen05/TMEM/TMA GEMM,
  FlashAttention forward/backward, int8 weight-only GEMM, column-parallel TP
  GEMM with NVLink peer stores) behind the C ABI of ``include/dgx.h``;
* ``libdream_b200.so`` — the Dream runtime's op signatures for this path
  (``tensor_matmul``, ``dream_linear``, ``dream_flash_attention``,
  ``dream_tp_matmul_column``, ``backward`` ...) forwarding into libdgx.

This Python module is a thin convenience layer over the C ABI for callers that
hold torch CUDA tensors (tests, bench). It never computes on the CPU.
"""
from __future__ import annotations

from . import _lib
from .ops import (  # noqa: F401
    gemm, bmm, gemm_batched, conv2d, conv2d_backward, flash_fwd_rows, flash_bwd_rows, flash_fwd, flash_bwd, gemm_w8, gemm_i8i32, quantize_rows_i8,
    gemm_workspace_size, flash_bwd_workspace_size, flash_set_deterministic, init, sync_check, version,
)
from ._lib import DgxError  # noqa: F401

__all__ = ["gemm", "bmm", "gemm_batched", "conv2d", "conv2d_backward", "flash_fwd_rows", "flash_bwd_rows", "flash_fwd", "flash_bwd", "gemm_w8", "gemm_i8i32", "quantize_rows_i8",
           "gemm_workspace_size", "flash_bwd_workspace_size", "flash_set_deterministic", "init", "sync_check",
           "version", "DgxError"]
