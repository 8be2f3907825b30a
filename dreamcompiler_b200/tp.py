"""Column-parallel tensor-parallel GEMM across processes (one per GPU).

Wraps dgx_tp_export / dgx_tp_open / dgx_tp_gemm_colsplit: every rank holds
all of A and its column shard of B (reference shard widths, see
dgx_tp_shard); after a call C_full on every rank holds A @ B. The IPC
handles are exchanged once through torch.distributed (any backend).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .ops import tp_shard  # noqa: F401

_DT = {torch.float32: L.DGX_F32, torch.bfloat16: L.DGX_BF16}


class ColumnParallelGemm:
    def __init__(self, M: int, N: int, K: int, rank: int, world: int, *, out_dtype=torch.bfloat16,
                 device=None, group=None):
        import torch.distributed as dist
        self.M, self.N, self.K, self.rank, self.world = M, N, K, rank, world
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.out_dtype = out_dtype
        self.C = torch.zeros(M, N, device=self.device, dtype=out_dtype)
        lib = L.load()
        hsz = lib.dgx_tp_handle_size()
        buf = (C.c_char * hsz)()
        L.call("dgx_tp_export", self.C.data_ptr(), self.C.numel() * self.C.element_size(), buf, hsz)
        mine = bytes(buf)
        if world > 1:
            got = [None] * world
            dist.all_gather_object(got, mine, group=group)
        else:
            got = [mine]
        allh = (C.c_char * (hsz * world)).from_buffer_copy(b"".join(got))
        L.call("dgx_tp_open", rank, world, allh)
        self.col0, self.ncol = tp_shard(N, world, rank)

    def __call__(self, A: torch.Tensor, B_shard: torch.Tensor, timeout_ms: int = 10000) -> torch.Tensor:
        assert A.is_contiguous() and B_shard.is_contiguous() and A.dtype == B_shard.dtype
        assert A.shape == (self.M, self.K) and B_shard.shape == (self.K, self.ncol)
        L.call("dgx_tp_gemm_colsplit", A.data_ptr(), B_shard.data_ptr(), self.M, self.N, self.K, _DT[A.dtype],
               _DT[self.out_dtype], timeout_ms, torch.cuda.current_stream(self.device).cuda_stream)
        return self.C

    def close(self) -> None:
        L.call("dgx_tp_close")
