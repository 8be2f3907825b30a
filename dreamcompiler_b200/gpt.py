"""Device-resident GPT training step on libdgx.

The model is the one a Dream program builds from the reference ops (see the
restatement in oracle/gpt_oracle.py): token + position embedding, L pre-LN
blocks of causal multi-head attention and a 4x GELU(tanh) MLP, a final
layer_norm, a linear head, log_softmax + nll_loss, and AdamW. Every `linear`
runs on dgx_gemm (bf16 operands, fp32 accumulate and bias epilogue), the
attention on dgx_flash_fwd_rows / dgx_flash_bwd_rows (heads read from and
written to token rows), everything else on the libdgx
device ops (dgx_layernorm_*, dgx_gelu_*, dgx_embedding_*, dgx_softmax_nll,
dgx_colsum, dgx_adamw, the head layout permutes). Parameters, gradients and
AdamW state are fp32; the GEMMs read bf16 copies of the weights refreshed
after each update. The residual stream and its gradient stay fp32; tensors
whose only consumers read bf16 (the QKV projection, the MLP pre-activation
and its gradient) are produced in bf16 by the GEMM epilogue.

All buffers are allocated up front, so one `step` can be captured in a CUDA
graph and replayed (the AdamW step count lives on the device).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict

import torch

from . import _lib as L
from .ops import _stream, flash_bwd_workspace_size, gemm


@dataclass
class GPTConfig:
    n_layer: int = 6
    d_model: int = 384
    n_head: int = 6
    seq_len: int = 256
    batch: int = 64
    vocab: int = 65
    lr: float = 3e-4
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.01

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head

    @property
    def vocab_pad(self) -> int:  # logits row pitch: 16-byte rows for the bf16 GEMM operand
        return (self.vocab + 7) // 8 * 8

    def n_params(self) -> int:
        d, L_ = self.d_model, self.n_layer
        return L_ * (12 * d * d + 9 * d) + (2 * self.vocab + self.seq_len) * d + self.vocab

    def flops_per_step(self) -> float:
        """Algorithmic FLOPs: 6 * (GEMM parameters) * tokens for the dense part
        plus causal attention forward (4*S^2*D/2 per head) and backward (2.5x)."""
        d, L_, S = self.d_model, self.n_layer, self.seq_len
        tokens = self.batch * S
        dense = 6 * (L_ * 12 * d * d + self.vocab * d) * tokens
        attn = L_ * self.batch * self.n_head * 3.5 * 4 * S * S * self.head_dim / 2
        return dense + attn


def _c(name, *args):
    L.call(name, *args)


class GPT:
    """Parameters, optimizer state and activations of one GPT on one GPU."""

    def __init__(self, cfg: GPTConfig, device="cuda", params: Dict[str, torch.Tensor] = None, seed: int = 0):
        self.cfg = c = cfg
        dev = self.dev = torch.device(device)
        d, H, hd, S, B, V, Vp = c.d_model, c.n_head, c.head_dim, c.seq_len, c.batch, c.vocab, c.vocab_pad
        assert d % H == 0 and hd % 8 == 0 and hd <= 64, "head_dim must be a multiple of 8, at most 64"
        R = self.R = B * S
        f32, bf16 = torch.float32, torch.bfloat16

        # ---- parameters: matrices (weight decay) and biases (none) in two flat buffers
        mats = {"W_tok": (V, d), "P": (S, d)}
        vecs = {}
        for l in range(c.n_layer):
            mats.update({f"Wqkv{l}": (3 * d, d), f"Wo{l}": (d, d), f"W1{l}": (4 * d, d), f"W2{l}": (d, 4 * d)})
            vecs.update({f"bqkv{l}": (3 * d,), f"bo{l}": (d,), f"b1{l}": (4 * d,), f"b2{l}": (d,)})
        mats["Wout"] = (Vp, d)
        vecs["bout"] = (Vp,)
        self.groups = {}
        self.p, self.g, self.w16 = {}, {}, {}
        for gname, spec in (("mat", mats), ("vec", vecs)):
            n = sum(torch.Size(s).numel() for s in spec.values())
            buf = {k: torch.zeros(n, device=dev, dtype=f32) for k in ("p", "g", "m", "v")}
            self.groups[gname] = buf
            if gname == "mat":
                self.w16_flat = torch.zeros(n, device=dev, dtype=bf16)
            off = 0
            for name, shp in spec.items():
                k = torch.Size(shp).numel()
                self.p[name] = buf["p"][off:off + k].view(shp)
                self.g[name] = buf["g"][off:off + k].view(shp)
                if gname == "mat":
                    self.w16[name] = self.w16_flat[off:off + k].view(shp)
                off += k
        self.step_dev = torch.zeros(1, device=dev, dtype=torch.int32)
        self._init(params, seed)

        # ---- activations kept for the backward
        self.tok = torch.zeros(R, device=dev, dtype=torch.int32)
        self.tgt = torch.zeros(R, device=dev, dtype=torch.int32)
        self.x = [torch.empty(R, d, device=dev, dtype=f32) for _ in range(2 * c.n_layer + 1)]
        self.h16 = [torch.empty(R, d, device=dev, dtype=bf16) for _ in range(2 * c.n_layer + 1)]
        self.mu = [torch.empty(R, device=dev, dtype=f32) for _ in range(2 * c.n_layer + 1)]
        self.rs = [torch.empty(R, device=dev, dtype=f32) for _ in range(2 * c.n_layer + 1)]
        # Q, K, V stay inside the QKV projection's token rows: the attention
        # kernels read heads there (dgx_flash_fwd_rows) and write O as rows.
        self.qkv16 = [torch.empty(R, 3 * d, device=dev, dtype=bf16) for _ in range(c.n_layer)]
        self.lse = [torch.empty(B * H, S, device=dev, dtype=f32) for _ in range(c.n_layer)]
        self.att16 = [torch.empty(R, d, device=dev, dtype=bf16) for _ in range(c.n_layer)]
        self.u16 = [torch.empty(R, 4 * d, device=dev, dtype=bf16) for _ in range(c.n_layer)]
        self.g16 = [torch.empty(R, 4 * d, device=dev, dtype=bf16) for _ in range(c.n_layer)]
        self.logits = torch.empty(R, Vp, device=dev, dtype=f32)
        self.dlogits = torch.empty(R, Vp, device=dev, dtype=bf16)
        self.loss = torch.zeros(1, device=dev, dtype=f32)
        # ---- backward scratch
        self.dx = torch.empty(R, d, device=dev, dtype=f32)
        self.dx16 = torch.empty(R, d, device=dev, dtype=bf16)
        self.dh = torch.empty(R, d, device=dev, dtype=f32)
        self.dg16 = torch.empty(R, 4 * d, device=dev, dtype=bf16)
        self.du16 = torch.empty(R, 4 * d, device=dev, dtype=bf16)
        self.dqkv16 = torch.empty(R, 3 * d, device=dev, dtype=bf16)
        self.datt16 = torch.empty(R, d, device=dev, dtype=bf16)
        self.fa_ws = torch.empty(flash_bwd_workspace_size(B * H, S, hd) // 4 + 1, device=dev, dtype=f32)

    # ------------------------------------------------------------ setup
    def _init(self, params, seed):
        if params is None:
            from_cpu = {}
            gen = torch.Generator().manual_seed(seed)
            for name, t in self.p.items():
                std = 0.02 if name[0] in "WP" else 0.0
                if name.startswith(("Wo", "W2")):
                    std = 0.02 / (2 * self.cfg.n_layer) ** 0.5
                from_cpu[name] = torch.randn(t.shape, generator=gen) * std
            params = from_cpu
        for name, t in self.p.items():
            src = torch.as_tensor(params[name], dtype=torch.float32)
            if name in ("Wout", "bout"):  # rows / entries past the vocabulary stay zero
                t.zero_()
                t[:src.shape[0]].copy_(src)
            else:
                t.copy_(src.reshape(t.shape))
        self._refresh_w16()

    def _refresh_w16(self):
        s = _stream(self.w16_flat)
        mat = self.groups["mat"]["p"]
        _c("dgx_convert", mat.data_ptr(), L.DGX_F32, self.w16_flat.data_ptr(), L.DGX_BF16, mat.numel(), 0, s)

    def set_batch(self, tok: torch.Tensor, tgt: torch.Tensor):
        self.tok.copy_(tok.reshape(-1), non_blocking=True)
        self.tgt.copy_(tgt.reshape(-1), non_blocking=True)

    # ------------------------------------------------------------ step
    def forward_backward(self):
        c = self.cfg
        d, H, hd, S, B, V, Vp, R = c.d_model, c.n_head, c.head_dim, c.seq_len, c.batch, c.vocab, c.vocab_pad, self.R
        s = _stream(self.x[0])
        p, g, w = self.p, self.g, self.w16
        # ---- forward
        _c("dgx_embedding_fwd", self.tok.data_ptr(), p["W_tok"].data_ptr(), p["P"].data_ptr(), self.x[0].data_ptr(),
           R, S, d, V, s)
        for l in range(c.n_layer):
            x0, x1, x2 = self.x[2 * l], self.x[2 * l + 1], self.x[2 * l + 2]
            h, h2 = self.h16[2 * l], self.h16[2 * l + 1]
            _c("dgx_layernorm_fwd", x0.data_ptr(), h.data_ptr(), self.mu[2 * l].data_ptr(), self.rs[2 * l].data_ptr(),
               R, d, s)
            qkv = self.qkv16[l]
            gemm(h, w[f"Wqkv{l}"], transB=True, out=qkv, bias=p[f"bqkv{l}"])
            qp = qkv.data_ptr()
            _c("dgx_flash_fwd_rows", qp, 3 * d, qp + 2 * d, 3 * d, qp + 4 * d, 3 * d, self.att16[l].data_ptr(), d,
               self.lse[l].data_ptr(), B, H, S, hd, hd ** -0.5, 1, s)
            x1.copy_(x0)
            gemm(self.att16[l], w[f"Wo{l}"], transB=True, out=x1, bias=p[f"bo{l}"], beta=1.0)  # x1 = x0 + att Wo^T + bo
            _c("dgx_layernorm_fwd", x1.data_ptr(), h2.data_ptr(), self.mu[2 * l + 1].data_ptr(),
               self.rs[2 * l + 1].data_ptr(), R, d, s)
            gemm(h2, w[f"W1{l}"], transB=True, out=self.u16[l], bias=p[f"b1{l}"])
            _c("dgx_gelu_fwd", self.u16[l].data_ptr(), L.DGX_BF16, self.g16[l].data_ptr(), self.u16[l].numel(), s)
            x2.copy_(x1)
            gemm(self.g16[l], w[f"W2{l}"], transB=True, out=x2, bias=p[f"b2{l}"], beta=1.0)
        xL, hf = self.x[2 * c.n_layer], self.h16[2 * c.n_layer]
        _c("dgx_layernorm_fwd", xL.data_ptr(), hf.data_ptr(), self.mu[-1].data_ptr(), self.rs[-1].data_ptr(), R, d, s)
        gemm(hf, w["Wout"], transB=True, out=self.logits, bias=p["bout"])
        _c("dgx_softmax_nll", self.logits.data_ptr(), Vp, V, self.tgt.data_ptr(), R, self.loss.data_ptr(),
           self.dlogits.data_ptr(), L.DGX_BF16, s)
        # ---- backward
        gemm(self.dlogits, w["Wout"], out=self.dh)                        # dhf = dlogits Wout
        gemm(self.dlogits, hf, transA=True, out=g["Wout"])                # dWout = dlogits^T hf
        _c("dgx_colsum", self.dlogits.data_ptr(), L.DGX_BF16, g["bout"].data_ptr(), R, Vp, 0, s)
        # each layer-norm backward also leaves bf16(dx) in dx16 for the next GEMMs
        _c("dgx_layernorm_bwd_x16", xL.data_ptr(), self.mu[-1].data_ptr(), self.rs[-1].data_ptr(),
           self.dh.data_ptr(), self.dx.data_ptr(), self.dx16.data_ptr(), R, d, 0, s)
        for l in reversed(range(c.n_layer)):
            x0, x1 = self.x[2 * l], self.x[2 * l + 1]
            h, h2 = self.h16[2 * l], self.h16[2 * l + 1]
            # MLP: x2 = x1 + gelu(h2 W1^T + b1) W2^T + b2
            gemm(self.dx16, w[f"W2{l}"], out=self.dg16)                   # dg = dx W2
            gemm(self.dx16, self.g16[l], transA=True, out=g[f"W2{l}"])     # dW2 = dx^T g
            _c("dgx_colsum", self.dx.data_ptr(), L.DGX_F32, g[f"b2{l}"].data_ptr(), R, d, 0, s)
            _c("dgx_gelu_bwd", self.u16[l].data_ptr(), L.DGX_BF16, self.dg16.data_ptr(), L.DGX_BF16,
               self.du16.data_ptr(), self.du16.numel(), s)
            gemm(self.du16, w[f"W1{l}"], out=self.dh)                     # dh2 = du W1
            gemm(self.du16, h2, transA=True, out=g[f"W1{l}"])              # dW1 = du^T h2
            _c("dgx_colsum", self.du16.data_ptr(), L.DGX_BF16, g[f"b1{l}"].data_ptr(), R, 4 * d, 0, s)
            _c("dgx_layernorm_bwd_x16", x1.data_ptr(), self.mu[2 * l + 1].data_ptr(), self.rs[2 * l + 1].data_ptr(),
               self.dh.data_ptr(), self.dx.data_ptr(), self.dx16.data_ptr(), R, d, 1, s)
            # attention: x1 = x0 + merge(attn(split(h Wqkv^T + bqkv))) Wo^T + bo
            gemm(self.dx16, w[f"Wo{l}"], out=self.datt16)                 # datt = dx Wo (bf16 rows)
            gemm(self.dx16, self.att16[l], transA=True, out=g[f"Wo{l}"])   # dWo = dx^T att
            _c("dgx_colsum", self.dx.data_ptr(), L.DGX_F32, g[f"bo{l}"].data_ptr(), R, d, 0, s)
            # dQ, dK, dV land in the dQKV rows the next GEMMs read
            qp, gp = self.qkv16[l].data_ptr(), self.dqkv16.data_ptr()
            _c("dgx_flash_bwd_rows", qp, 3 * d, qp + 2 * d, 3 * d, qp + 4 * d, 3 * d, self.att16[l].data_ptr(), d,
               self.datt16.data_ptr(), d, self.lse[l].data_ptr(), gp, 3 * d, gp + 2 * d, 3 * d, gp + 4 * d, 3 * d,
               B, H, S, hd, hd ** -0.5, 1, self.fa_ws.data_ptr(), self.fa_ws.numel() * 4, s)
            gemm(self.dqkv16, w[f"Wqkv{l}"], out=self.dh)                 # dh = dqkv Wqkv
            gemm(self.dqkv16, h, transA=True, out=g[f"Wqkv{l}"])           # dWqkv = dqkv^T h
            _c("dgx_colsum", self.dqkv16.data_ptr(), L.DGX_BF16, g[f"bqkv{l}"].data_ptr(), R, 3 * d, 0, s)
            if l > 0:
                _c("dgx_layernorm_bwd_x16", x0.data_ptr(), self.mu[2 * l].data_ptr(), self.rs[2 * l].data_ptr(),
                   self.dh.data_ptr(), self.dx.data_ptr(), self.dx16.data_ptr(), R, d, 1, s)
            else:  # the embedding backward reads dx in fp32 only
                _c("dgx_layernorm_bwd", x0.data_ptr(), self.mu[2 * l].data_ptr(), self.rs[2 * l].data_ptr(),
                   self.dh.data_ptr(), self.dx.data_ptr(), R, d, 1, s)
        g["W_tok"].zero_()
        g["P"].zero_()
        _c("dgx_embedding_bwd", self.tok.data_ptr(), self.dx.data_ptr(), g["W_tok"].data_ptr(), g["P"].data_ptr(),
           R, S, d, V, s)
        return self.loss

    def optimizer_step(self):
        c = self.cfg
        s = _stream(self.step_dev)
        self.step_dev.add_(1)
        for gname, wd in (("mat", c.weight_decay), ("vec", 0.0)):
            b = self.groups[gname]
            _c("dgx_adamw", b["p"].data_ptr(), b["g"].data_ptr(), b["m"].data_ptr(), b["v"].data_ptr(), b["p"].numel(),
               c.lr, c.betas[0], c.betas[1], c.eps, wd, 0, self.step_dev.data_ptr(), s)
        self._refresh_w16()

    def step(self):
        loss = self.forward_backward()
        self.optimizer_step()
        return loss
