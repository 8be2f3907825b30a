"""TEST INFRASTRUCTURE: timed CPU runs of the hot path for bench.py's
cpu_baseline and `--impl reference` arm. Imports no torch, so spawned worker
processes start in well under a second.

The reference path is the reference runtime compiled from its own sources
(oracle/_ref/libdream_ref.so) driven through its C ABI, exactly the calls a
Dream program makes: flash_attention(Q, K, V, B, S, dk, 64) followed by
backward(). When that library is absent the CPU restatement (liboracle.so)
stands in and the result says kind "port".
"""
from __future__ import annotations

import os
import time


def flash_head(kind: str, seed: int, S: int, dk: int) -> float:
    """Seconds for one head's causal FlashAttention forward + backward."""
    if kind == "reference":
        from oracle import refrt as R
        R.set_seed(seed)
        Q, K, V = (R.randn(1, S * dk) for _ in range(3))
        sc = [R.scalar(v) for v in (1, S, dk, 64)]
        t0 = time.perf_counter()
        O = R.call("dream_flash_attention", Q, K, V, *sc)
        R.call("backward", O)  # seeds dO = 1 (autograd.inc:34); same work as any dO
        return time.perf_counter() - t0
    from oracle import orc
    orc.set_seed(seed)
    Q, K, V = (orc.randn(1, S, dk) for _ in range(3))
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    t0 = time.perf_counter()
    O, _ = orc.flash_fwd(Q, K, V)
    orc.flash_bwd(Q, K, V, O * 0 + 1)
    return time.perf_counter() - t0


def gemm_rows(kind: str, seed: int, n: int, rows: int) -> float:
    """Seconds for `rows` rows of an n^3 f64 GEMM (dream_gemm_d semantics)."""
    from oracle import orc
    import numpy as np
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((rows, n))
    B = rng.standard_normal((n, n))
    t0 = time.perf_counter()
    orc.gemm_f64(A, B)
    return time.perf_counter() - t0


def available_kind() -> str:
    from oracle import refrt
    return "reference" if refrt.available() else "port"
