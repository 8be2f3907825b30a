"""Profiling entry point: run one small case of a hot-path kernel through the
C ABI, sized for an `ncu` capture (a few hundred MB on the device at most,
two launches of each kernel).

    python -m dreamcompiler_b200.profile_case flash --bh 16      # S=2048, D=64
    python -m dreamcompiler_b200.profile_case gemm --n 4096
    python -m dreamcompiler_b200.profile_case w8 --batch 1 --mode 1   # int8 layer, N=K=4096
    python -m dreamcompiler_b200.profile_case gemm_f32 --n 1024       # 3xTF32
    python -m dreamcompiler_b200.profile_case conv --batch 8          # 64 -> 128 channels, 3x3, 32x32
    python -m dreamcompiler_b200.profile_case gpt                     # one config-3 training step
    python -m dreamcompiler_b200.profile_case linear                  # GPT MLP-up: 16384x1536x384 + bias
    python -m dreamcompiler_b200.profile_case gemm_f64 --n 4096       # f64 DFMA GEMM
"""
from __future__ import annotations

import argparse


def main() -> None:
    import torch
    import dreamcompiler_b200 as dgx

    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["flash", "gemm", "w8", "gemm_f32", "conv", "gpt", "linear", "gemm_f64"])
    ap.add_argument("--bh", type=int, default=16)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--mode", type=int, default=0, help="w8: 0 = W8A32, 1 = W8A8")
    ap.add_argument("--reps", type=int, default=2)
    a = ap.parse_args()
    dgx.init(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.kind == "flash":
        Q, K, V, dO = (torch.randn(a.bh, a.seq, a.dim, device="cuda", generator=g).bfloat16() for _ in range(4))
        O, L = dgx.flash_fwd(Q, K, V)
        for _ in range(a.reps):
            dgx.flash_fwd(Q, K, V, out=O, lse=L)
            dgx.flash_bwd(Q, K, V, O, dO, L)
    elif a.kind == "gemm":
        A, B = (torch.randn(a.n, a.n, device="cuda", generator=g).bfloat16() for _ in range(2))
        C = torch.empty(a.n, a.n, device="cuda", dtype=torch.bfloat16)
        for _ in range(a.reps):
            dgx.gemm(A, B, out=C)
    elif a.kind == "linear":  # X.W^T + b at the GPT step's MLP-up shape (bf16 out)
        X = torch.randn(16384, 384, device="cuda", generator=g).bfloat16()
        W = (torch.randn(1536, 384, device="cuda", generator=g) / 384 ** 0.5).bfloat16()
        b = torch.randn(1536, device="cuda", generator=g)
        Y = torch.empty(16384, 1536, device="cuda", dtype=torch.bfloat16)
        for _ in range(a.reps):
            dgx.gemm(X, W, transB=True, out=Y, bias=b)
    elif a.kind == "gemm_f32":
        A, B, dC = (torch.randn(a.n, a.n, device="cuda", generator=g) for _ in range(3))
        for _ in range(a.reps):
            dgx.gemm(A, B)
            dgx.gemm(dC, B, transB=True)
            dgx.gemm(A, dC, transA=True)
    elif a.kind == "conv":
        X = torch.randn(a.batch, 64, 32, 32, device="cuda", generator=g)
        Kw = torch.randn(128, 64 * 9, device="cuda", generator=g) / 24.0
        b = torch.randn(128, device="cuda", generator=g)
        for _ in range(a.reps):
            Y = dgx.conv2d(X, Kw, b, 3, 3, pad=1, operands=torch.bfloat16)
            dgx.conv2d_backward(X, Kw, Y, 3, 3, pad=1, operands=torch.bfloat16)
    elif a.kind == "gemm_f64":
        A, B = (torch.randn(a.n, a.n, device="cuda", generator=g, dtype=torch.float64) for _ in range(2))
        for _ in range(a.reps):
            dgx.gemm(A, B)
    elif a.kind == "gpt":
        from dreamcompiler_b200.gpt import GPT, GPTConfig
        cfg = GPTConfig()
        model = GPT(cfg, device="cuda", seed=0)
        gt = torch.Generator().manual_seed(3)
        tok = torch.randint(0, cfg.vocab, (cfg.batch * cfg.seq_len,), generator=gt, dtype=torch.int32)
        model.set_batch(tok, torch.randint(0, cfg.vocab, tok.shape, generator=gt, dtype=torch.int32))
        for _ in range(a.reps):
            model.step()
    else:
        X = torch.randn(a.batch, a.n, device="cuda", generator=g)
        W = torch.randint(-127, 128, (a.n, a.n), device="cuda", dtype=torch.int8, generator=g)
        sc = torch.rand(a.n, device="cuda", generator=g) * 9e-3 + 1e-3
        for _ in range(a.reps):
            dgx.gemm_w8(X, W, sc, None, mode=a.mode)
    dgx.sync_check()
    print("profile case ok")


if __name__ == "__main__":
    main()
