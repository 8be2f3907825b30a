"""Torch-tensor wrappers over the libdgx C ABI.

Each function validates dtypes/devices, passes raw device pointers and the
current torch CUDA stream to the C entry point, and raises ``DgxError`` on a
non-OK status. Outputs are allocated with torch when not supplied.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib as L

_DT = {torch.float32: L.DGX_F32, torch.bfloat16: L.DGX_BF16, torch.int8: L.DGX_I8}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def version() -> str:
    return L.load().dgx_version().decode()


def init(device: int = 0) -> None:
    L.call("dgx_init", device)


def sync_check(stream: Optional[int] = None) -> None:
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    L.call("dgx_sync_check", stream)


def gemm_workspace_size(M, N, K, transA=False, transB=False, dtype=torch.float32, f32_mode=0) -> int:
    return L.load().dgx_gemm_workspace_size(M, N, K, int(transA), int(transB), _DT[dtype], f32_mode)


def gemm(A: torch.Tensor, B: torch.Tensor, *, transA: bool = False, transB: bool = False,
         out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
         bias: Optional[torch.Tensor] = None, relu: bool = False, beta: float = 0.0,
         f32_mode: int = L.DGX_F32_3XTF32, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = beta*C + op(A) @ op(B) (+bias) (ReLU). A, B: 2-D row-major CUDA tensors,
    possibly with a row pitch (stride(0)) larger than their width. float64
    operands run the f64 kernel (dgx_gemm_f64) with an f64 result and bias."""
    assert A.is_cuda and B.is_cuda and A.dtype == B.dtype and A.dim() == 2 and B.dim() == 2
    assert A.stride(1) == 1 and B.stride(1) == 1, "inner dimension must be contiguous"
    M, K = (A.shape[1], A.shape[0]) if transA else (A.shape[0], A.shape[1])
    Kb, N = (B.shape[1], B.shape[0]) if transB else (B.shape[0], B.shape[1])
    assert K == Kb, f"inner dimensions differ: {K} vs {Kb}"
    if A.dtype == torch.float64:
        if out is None:
            out = torch.empty(M, N, device=A.device, dtype=torch.float64)
        assert out.dtype == torch.float64 and out.stride(1) == 1 and out.shape == (M, N)
        epi = L.DGX_EPI_NONE
        if bias is not None:
            assert bias.dtype == torch.float64 and bias.is_contiguous() and bias.numel() == N
            epi = L.DGX_EPI_BIAS_RELU if relu else L.DGX_EPI_BIAS
        elif relu:
            epi = L.DGX_EPI_RELU
        L.call("dgx_gemm_f64", A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, A.stride(0), B.stride(0),
               out.stride(0), int(transA), int(transB), _ptr(bias), epi, float(beta), _stream(A))
        return out
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=out_dtype or torch.float32)
    assert out.stride(1) == 1 and out.shape == (M, N)
    epi = L.DGX_EPI_NONE
    if bias is not None:
        assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == N
        epi = L.DGX_EPI_BIAS_RELU if relu else L.DGX_EPI_BIAS
    elif relu:
        epi = L.DGX_EPI_RELU
    ws, wsb = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    L.call("dgx_gemm", A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, A.stride(0), B.stride(0),
           out.stride(0), int(transA), int(transB), _DT[A.dtype], _DT[out.dtype], f32_mode, _ptr(bias), epi,
           float(beta), ws, wsb, _stream(A))
    return out


def bmm(A: torch.Tensor, B: torch.Tensor, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    assert A.dim() == 3 and B.dim() == 3 and A.is_contiguous() and B.is_contiguous()
    batch, M, K = A.shape
    N = B.shape[2]
    out = torch.empty(batch, M, N, device=A.device, dtype=out_dtype)
    L.call("dgx_bmm", A.data_ptr(), B.data_ptr(), out.data_ptr(), batch, M, N, K, _DT[A.dtype], _DT[out_dtype],
           _stream(A))
    return out


def gemm_batched(A: torch.Tensor, B: torch.Tensor, *, transA: bool = False, transB: bool = False,
                 out: Optional[torch.Tensor] = None, beta: float = 0.0,
                 out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """C[b] = op(A[b]) . op(B[b]) (+ beta*C[b]) for 3-D tensors whose last dim
    is contiguous (any batch and row strides); one launch for all batches."""
    assert A.dim() == 3 and B.dim() == 3 and A.dtype == B.dtype
    assert A.stride(2) == 1 and B.stride(2) == 1
    batch = A.shape[0]
    M, K = (A.shape[2], A.shape[1]) if transA else (A.shape[1], A.shape[2])
    N = B.shape[1] if transB else B.shape[2]
    assert B.shape[0] == batch and (B.shape[2] if transB else B.shape[1]) == K
    if out is None:
        out = torch.empty(batch, M, N, device=A.device, dtype=out_dtype)
    assert out.shape == (batch, M, N) and out.stride(2) == 1
    L.call("dgx_gemm_batched", A.data_ptr(), B.data_ptr(), out.data_ptr(), batch, M, N, K, A.stride(1),
           B.stride(1), out.stride(1), A.stride(0), B.stride(0), out.stride(0), int(transA), int(transB),
           _DT[A.dtype], _DT[out.dtype], float(beta), _stream(A))
    return out


def flash_fwd_rows(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, O: torch.Tensor, lse: torch.Tensor,
                   B: int, H: int, S: int, D: int, *, causal: bool = True, scale: Optional[float] = None) -> None:
    """FlashAttention forward on heads inside token rows: Q, K, V, O are 2-D
    bf16 views [B*S, >= H*D] (column slices of one buffer allowed, e.g.
    qkv[:, 0:HD], qkv[:, HD:2HD], qkv[:, 2HD:]); head h is columns
    [h*D, (h+1)*D). lse: [B*H, S] fp32."""
    for t in (Q, K, V, O):
        assert t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1
    L.call("dgx_flash_fwd_rows", Q.data_ptr(), Q.stride(0), K.data_ptr(), K.stride(0), V.data_ptr(), V.stride(0),
           O.data_ptr(), O.stride(0), lse.data_ptr(), B, H, S, D, D ** -0.5 if scale is None else scale,
           int(causal), _stream(Q))


def flash_bwd_rows(Q, K, V, O, dO, lse, dQ, dK, dV, B: int, H: int, S: int, D: int, *, causal: bool = True,
                   scale: Optional[float] = None, workspace: Optional[torch.Tensor] = None) -> None:
    """Backward of flash_fwd_rows; dQ, dK, dV are row views like Q, K, V."""
    for t in (Q, K, V, O, dO, dQ, dK, dV):
        assert t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1
    ws, wsb = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    L.call("dgx_flash_bwd_rows", Q.data_ptr(), Q.stride(0), K.data_ptr(), K.stride(0), V.data_ptr(), V.stride(0),
           O.data_ptr(), O.stride(0), dO.data_ptr(), dO.stride(0), lse.data_ptr(), dQ.data_ptr(), dQ.stride(0),
           dK.data_ptr(), dK.stride(0), dV.data_ptr(), dV.stride(0), B, H, S, D, D ** -0.5 if scale is None else scale,
           int(causal), ws, wsb, _stream(Q))


def conv2d(X: torch.Tensor, Kw: torch.Tensor, bias: Optional[torch.Tensor], KH: int, KW: int, *, pad: int = 0,
           stride: int = 1, operands: torch.dtype = torch.float32) -> torch.Tensor:
    """X [N, Cin, H, W] fp32, Kw [Cout, Cin*KH*KW] fp32 (row per output
    channel), bias [Cout] or None -> Y [N, Cout, OH, OW] fp32. `operands`
    float32 runs 3xTF32 GEMMs, bfloat16 bf16 ones."""
    assert X.dtype == torch.float32 and Kw.dtype == torch.float32 and X.is_contiguous() and Kw.is_contiguous()
    N, Cin, H, W = X.shape
    Cout = Kw.shape[0]
    OH, OW = (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1
    Y = torch.empty(N, Cout, OH, OW, device=X.device, dtype=torch.float32)
    L.call("dgx_conv2d_fwd", X.data_ptr(), Kw.data_ptr(), _ptr(bias), Y.data_ptr(), N, Cin, H, W, Cout, KH, KW, pad,
           stride, _DT[operands], _stream(X))
    return Y


def conv2d_backward(X: torch.Tensor, Kw: torch.Tensor, dY: torch.Tensor, KH: int, KW: int, *, pad: int = 0,
                    stride: int = 1, operands: torch.dtype = torch.float32):
    """(dX, dK) of conv2d for the output gradient dY [N, Cout, OH, OW]."""
    N, Cin, H, W = X.shape
    Cout = Kw.shape[0]
    dX = torch.empty_like(X)
    dK = torch.empty_like(Kw)
    L.call("dgx_conv2d_bwd", X.data_ptr(), Kw.data_ptr(), dY.contiguous().data_ptr(), dX.data_ptr(), dK.data_ptr(),
           N, Cin, H, W, Cout, KH, KW, pad, stride, _DT[operands], 0, _stream(X))
    return dX, dK


def flash_fwd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, causal: bool = True,
              scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
              lse: Optional[torch.Tensor] = None, want_lse: bool = True):
    """Q, K, V: [BH, S, D] bf16 contiguous. Returns (O, LSE)."""
    assert Q.dtype == torch.bfloat16 and Q.is_contiguous() and K.is_contiguous() and V.is_contiguous()
    BH, S, D = Q.shape
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty_like(Q)
    if lse is None and want_lse:
        lse = torch.empty(BH, S, device=Q.device, dtype=torch.float32)
    L.call("dgx_flash_fwd", Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), _ptr(lse), BH, S, D,
           float(scale), int(causal), L.DGX_BF16, _stream(Q))
    return out, lse


def flash_set_deterministic(on: bool) -> None:
    """Process-wide: backward calls with D <= 64 take the two-kernel form
    (every gradient bit-reproducible) instead of the one-kernel form."""
    L.call("dgx_flash_set_deterministic", int(bool(on)))


def flash_bwd_workspace_size(BH: int, S: int, D: int) -> int:
    return L.load().dgx_flash_bwd_workspace_size(BH, S, D)


def flash_bwd(Q, K, V, O, dO, lse, *, causal: bool = True, scale: Optional[float] = None,
              dQ=None, dK=None, dV=None, workspace: Optional[torch.Tensor] = None):
    BH, S, D = Q.shape
    if scale is None:
        scale = D ** -0.5
    dQ = torch.empty_like(Q) if dQ is None else dQ
    dK = torch.empty_like(K) if dK is None else dK
    dV = torch.empty_like(V) if dV is None else dV
    ws, wsb = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    L.call("dgx_flash_bwd", Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), dO.data_ptr(), lse.data_ptr(),
           dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), BH, S, D, float(scale), int(causal), L.DGX_BF16, ws, wsb,
           _stream(Q))
    return dQ, dK, dV


def gemm_w8(X: torch.Tensor, W: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
            mode: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """X [B,K] fp32, W [N,K] int8, scale [N] fp32 -> Y [B,N] fp32."""
    assert X.dtype == torch.float32 and W.dtype == torch.int8 and scale.dtype == torch.float32
    B, K = X.shape
    N = W.shape[0]
    if out is None:
        out = torch.empty(B, N, device=X.device, dtype=torch.float32)
    L.call("dgx_gemm_w8", X.data_ptr(), W.data_ptr(), scale.data_ptr(), _ptr(bias), out.data_ptr(), B, N, K, mode,
           _stream(X))
    return out


def gemm_i8i32(Xq: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    B, K = Xq.shape
    N = W.shape[0]
    acc = torch.empty(B, N, device=Xq.device, dtype=torch.int32)
    L.call("dgx_gemm_i8i32", Xq.data_ptr(), W.data_ptr(), acc.data_ptr(), B, N, K, _stream(Xq))
    return acc


def quantize_rows_i8(X: torch.Tensor):
    B, K = X.shape
    Xq = torch.empty(B, K, device=X.device, dtype=torch.int8)
    sx = torch.empty(B, device=X.device, dtype=torch.float32)
    L.call("dgx_quantize_rows_i8", X.data_ptr(), Xq.data_ptr(), sx.data_ptr(), B, K, _stream(X))
    return Xq, sx


def tp_shard(N: int, world: int, rank: int):
    col0, ncol = C.c_int(0), C.c_int(0)
    L.load().dgx_tp_shard(N, world, rank, C.byref(col0), C.byref(ncol))
    return col0.value, ncol.value
