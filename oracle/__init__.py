"""TEST INFRASTRUCTURE — the CPU checker for the hot path, never the product.

* ``oracle.orc``   — ctypes binding of liboracle.so, this repository's CPU
  restatement of the reference arithmetic (dream_oracle.cpp).
* ``oracle.refrt`` — ctypes binding of oracle/_ref/libdream_ref.so, the
  reference Dream runtime compiled from its own sources (build_ref.sh).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this package.
"""
