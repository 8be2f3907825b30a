"""Generate the golden vectors in tests/golden/ from the reference runtime.

Runs only where the reference sources exist (it loads
oracle/_ref/libdream_ref.so, built by oracle/build_ref.sh from
heellowdsf/DreamCompiler runtime/). Every input is drawn with the reference's
own RNG (set_seed + randn, runtime/ops/elementwise.inc:30-55) and every
output comes from the reference's own ops:

  gemm.npz   tensor_matmul f64 and f32-mirror paths + "matmul" backward, on
             the shapes of gemm_selftest (runtime/ops/elementwise.inc:893-896)
  flash.npz  dream_flash_attention + its backward, dream_attention_causal,
             on the flash_attention_selftest configs (runtime/nn/training.inc:411)
             and the tests/26_flash_backward.dream case
  linear.npz dream_linear / dream_linear_relu + backward
  tp.npz     dream_tp_matmul_column for G in {2,3,4,5,7} (training.inc:1664-1706)
  gpt.npz    one GPT training step (BASELINE config 3 architecture at a tiny
             size) composed from the reference ops: embedding + broadcast
             position add, layer_norm, per-head dream_linear and
             dream_flash_attention, gelu, log_softmax + nll_loss, backward;
             parameters from a seeded numpy generator (oracle/gpt_oracle.py)
  adamw.npz  dream_adamw_update applied twice to one parameter
  bmm.npz    dream_bmm + its "bmm" backward (runtime/ops/elementwise.inc:1218-1252,
             runtime/ops/autograd.inc:549-574)
  attn.npz   dream_attention and dream_attention_causal + their backward
             (runtime/nn/training.inc:177-263, runtime/ops/autograd.inc:675-778)
  conv.npz   dream_conv2d + its "conv2d" backward, dream_conv2d_padded forward
             (runtime/nn/conv.inc:12-187, runtime/ops/autograd.inc:507-535)
  int8_export/mlp_int8.{c,h} + int8_export.npz
             a 3-layer MLP checkpoint exported by the reference's own
             export_c_header_int8 (runtime/nn/training.inc:3494-3817); inputs
             X and the outputs Y of that emitted C code (compiled with cc),
             plus Ypc from the per-channel variant this repository writes
             (dreamcompiler_b200/int8_export.py) for the same weights

Usage:  python tests/golden/make_golden.py [fixture ...]
"""
from __future__ import annotations

import ctypes as C
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import refrt as R  # noqa: E402

# gemm_selftest's shapes up to 128x100x96 (its two largest are left out to keep the fixture small)
GEMM_SHAPES = [(1, 1, 1), (1, 7, 1), (5, 1, 9), (3, 4, 5), (7, 13, 17), (31, 33, 37), (64, 64, 64), (65, 63, 66),
               (128, 100, 96)]
FLASH_CFGS = [(64, 16, 8), (64, 16, 16), (128, 32, 32), (100, 24, 16), (128, 64, 64), (160, 64, 32)]


def seeded_backward(out, shape):
    """backward(sum(out * G)) with G ~ randn: injects dOut = G (autograd.inc:26)."""
    g = R.randn(*shape)
    s = R.call("sum", R.call("tensor_mul", out, g))
    R.call("backward", s)
    return R.data(g)


def gen_gemm():
    out = {}
    R.set_seed(42)
    for (M, K, N) in GEMM_SHAPES:
        A, B = R.randn(M, K), R.randn(K, N)
        C = R.call("tensor_matmul", A, B)
        G = seeded_backward(C, (M, N))
        tag = f"{M}x{K}x{N}"
        out[f"A_{tag}"], out[f"B_{tag}"], out[f"G_{tag}"] = R.data(A), R.data(B), G
        out[f"C_{tag}"], out[f"dA_{tag}"], out[f"dB_{tag}"] = R.data(C), R.grad(A), R.grad(B)
        # f32 mirror path: dream_set_precision(t, 1) then `@` (elementwise.inc:1000-1016)
        A32, B32 = R.tensor(out[f"A_{tag}"]), R.tensor(out[f"B_{tag}"])
        R.call("dream_set_precision", A32, 1)
        R.call("dream_set_precision", B32, 1)
        out[f"C32_{tag}"] = R.data(R.call("tensor_matmul", A32, B32))
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **out)


def gen_flash():
    out = {}
    R.set_seed(20260709)
    for (S, dk, Bc) in FLASH_CFGS:
        B = 2 if S * dk <= 4096 else 1
        Q, K, V = R.randn(B, S * dk), R.randn(B, S * dk), R.randn(B, S * dk)
        sc = [R.scalar(v) for v in (B, S, dk, Bc)]
        O = R.call("dream_flash_attention", Q, K, V, *sc)
        G = seeded_backward(O, (B, S * dk))
        tag = f"{S}_{dk}_{Bc}"
        for name, t in (("Q", Q), ("K", K), ("V", V)):
            out[f"{name}_{tag}"] = R.data(t).reshape(B, S, dk)
            out[f"d{name}_{tag}"] = R.grad(t).reshape(B, S, dk)
        out[f"G_{tag}"] = G.reshape(B, S, dk)
        out[f"O_{tag}"] = R.data(O).reshape(B, S, dk)
        Oc = R.call("dream_attention_causal", Q, K, V, *sc[:3])
        out[f"Ocausal_{tag}"] = R.data(Oc).reshape(B, S, dk)
        On = R.call("dream_attention", Q, K, V, *sc[:3])
        out[f"Ofull_{tag}"] = R.data(On).reshape(B, S, dk)
    # tests/26_flash_backward.dream: set_seed(5); Q,K,V = randn(1,512); S=32, dk=16, block 8; backward(sum(o)).
    R.set_seed(5)
    Q, K, V = R.randn(1, 512), R.randn(1, 512), R.randn(1, 512)
    O = R.call("dream_flash_attention", Q, K, V, R.scalar(1), R.scalar(32), R.scalar(16), R.scalar(8))
    R.call("backward", R.call("sum", O))
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        out[f"t26_{name}"] = R.data(t).reshape(1, 32, 16)
        out[f"t26_d{name}"] = R.grad(t).reshape(1, 32, 16)
    out["t26_O"] = R.data(O).reshape(1, 32, 16)
    np.savez_compressed(os.path.join(HERE, "flash.npz"), **out)


def gen_linear():
    out = {}
    R.set_seed(11)
    for relu in (0, 1):
        for (N, din, dout) in [(8, 16, 12), (33, 65, 17)]:
            X, W, b = R.randn(N, din), R.randn(dout, din), R.randn(1, dout)
            Y = R.call("dream_linear_relu" if relu else "dream_linear", X, W, b)
            G = seeded_backward(Y, (N, dout))
            tag = f"{relu}_{N}_{din}_{dout}"
            out[f"X_{tag}"], out[f"W_{tag}"], out[f"b_{tag}"], out[f"G_{tag}"] = R.data(X), R.data(W), R.data(b)[0], G
            out[f"Y_{tag}"], out[f"dX_{tag}"], out[f"dW_{tag}"], out[f"db_{tag}"] = (
                R.data(Y), R.grad(X), R.grad(W), R.grad(b)[0])
    np.savez_compressed(os.path.join(HERE, "linear.npz"), **out)


def gen_tp():
    out = {}
    R.set_seed(20260709)
    for (M, K, N) in [(12, 16, 24), (9, 10, 23)]:
        X, W = R.randn(M, K), R.randn(K, N)
        out[f"X_{M}_{K}_{N}"], out[f"W_{M}_{K}_{N}"] = R.data(X), R.data(W)
        for G in (1, 2, 3, 4, 5, 7):
            out[f"Y_{M}_{K}_{N}_{G}"] = R.data(R.call("dream_tp_matmul_column", X, W, R.scalar(G)))
    np.savez_compressed(os.path.join(HERE, "tp.npz"), **out)


GPT_CFG = dict(L=1, d=64, H=2, B=2, S=64, V=65, seed=3)


def gen_gpt():
    from oracle import gpt_oracle as G

    c = GPT_CFG
    L, d, H, B, S, V = c["L"], c["d"], c["H"], c["B"], c["S"], c["V"]
    hd, n = d // H, B * S
    params = G.init_params(L, d, V, S, c["seed"])
    rng = np.random.default_rng(c["seed"] + 1)
    tok = rng.integers(0, V, n)
    tgt = rng.integers(0, V, n)
    sc = R.scalar
    t = lambda a: R.tensor(np.asarray(a, np.float64).reshape(a.shape[0], -1) if a.ndim > 1 else
                           np.asarray(a, np.float64).reshape(1, -1))
    leaves = {}

    def leaf(name, a):
        leaves[name] = t(a)
        return leaves[name]

    e = R.call("dream_embedding", R.tensor(tok.astype(np.float64).reshape(n, 1)), leaf("W_tok", params["W_tok"]))
    pos = R.call("dream_reshape_nd", leaf("P", params["P"]), sc(1), sc(S * d))
    x = R.call("dream_reshape_nd", R.call("tensor_add", R.call("dream_reshape_nd", e, sc(B), sc(S * d)), pos),
               sc(n), sc(d))
    for l in range(L):
        h = R.call("dream_layer_norm", x)
        Wqkv, bqkv, Wo = params[f"Wqkv{l}"], params[f"bqkv{l}"], params[f"Wo{l}"]
        z = None
        for hh in range(H):
            qkv = []
            for i, nm in enumerate("qkv"):
                rows = slice(i * d + hh * hd, i * d + (hh + 1) * hd)
                y = R.call("dream_linear", h, leaf(f"W{nm}{l}_{hh}", Wqkv[rows]), leaf(f"b{nm}{l}_{hh}", bqkv[rows]))
                qkv.append(R.call("dream_reshape_nd", y, sc(B), sc(S * hd)))
            o = R.call("dream_flash_attention", *qkv, sc(B), sc(S), sc(hd), sc(64))
            o = R.call("dream_reshape_nd", o, sc(n), sc(hd))
            bias = params[f"bo{l}"] if hh == 0 else np.zeros(d, np.float32)
            zz = R.call("dream_linear", o, leaf(f"Wo{l}_{hh}", Wo[:, hh * hd:(hh + 1) * hd]), leaf(f"bo{l}_{hh}", bias))
            z = zz if z is None else R.call("tensor_add", z, zz)
        x = R.call("tensor_add", x, z)
        h2 = R.call("dream_layer_norm", x)
        u = R.call("dream_linear", h2, leaf(f"W1{l}", params[f"W1{l}"]), leaf(f"b1{l}", params[f"b1{l}"]))
        z2 = R.call("dream_linear", R.call("dream_gelu", u), leaf(f"W2{l}", params[f"W2{l}"]),
                    leaf(f"b2{l}", params[f"b2{l}"]))
        x = R.call("tensor_add", x, z2)
    hf = R.call("dream_layer_norm", x)
    logits = R.call("dream_linear", hf, leaf("Wout", params["Wout"]), leaf("bout", params["bout"]))
    loss = R.call("dream_nll_loss", R.call("dream_log_softmax", logits), R.tensor(tgt.astype(np.float64).reshape(n, 1)))
    R.call("backward", loss)

    grads = {}
    for name in ("W_tok", "P", "Wout", "bout"):
        grads[name] = R.grad(leaves[name]).reshape(params[name].shape)
    for l in range(L):
        for name in ("W1", "b1", "W2", "b2"):
            grads[f"{name}{l}"] = R.grad(leaves[f"{name}{l}"]).reshape(params[f"{name}{l}"].shape)
        gW = np.zeros((3 * d, d))
        gb = np.zeros(3 * d)
        gWo = np.zeros((d, d))
        for hh in range(H):
            for i, nm in enumerate("qkv"):
                rows = slice(i * d + hh * hd, i * d + (hh + 1) * hd)
                gW[rows] = R.grad(leaves[f"W{nm}{l}_{hh}"]).reshape(hd, d)
                gb[rows] = R.grad(leaves[f"b{nm}{l}_{hh}"]).reshape(hd)
            gWo[:, hh * hd:(hh + 1) * hd] = R.grad(leaves[f"Wo{l}_{hh}"]).reshape(d, hd)
        grads[f"Wqkv{l}"], grads[f"bqkv{l}"], grads[f"Wo{l}"] = gW, gb, gWo
        grads[f"bo{l}"] = R.grad(leaves[f"bo{l}_0"]).reshape(d)
    out = {"tok": tok.astype(np.int32), "tgt": tgt.astype(np.int32), "loss": np.float64(R.data(loss)[0, 0])}
    for k, v in params.items():
        out["p_" + k] = v
        out["g_" + k] = grads[k].astype(np.float32)
    out["cfg"] = np.array([c[k] for k in ("L", "d", "H", "B", "S", "V", "seed")], np.int64)
    np.savez_compressed(os.path.join(HERE, "gpt.npz"), **out)


def gen_adamw():
    rng = np.random.default_rng(11)
    p0 = rng.standard_normal((4, 50))
    g1, g2 = rng.standard_normal((4, 50)), rng.standard_normal((4, 50)) * 0.1
    p = R.tensor(p0)
    out = {"p0": p0, "g1": g1, "g2": g2}
    for k, g in enumerate((g1, g2), 1):
        C.memmove(p.contents.grad, np.ascontiguousarray(g, np.float64).ctypes.data, g.nbytes)
        R.call("dream_adamw_update", p, R.scalar(3e-4), R.scalar(0.9), R.scalar(0.999), R.scalar(1e-8), R.scalar(0.01))
        out[f"p{k}"] = R.data(p)
    np.savez_compressed(os.path.join(HERE, "adamw.npz"), **out)


# (batch, M, K, N) and (B, S, dk); stored as float32 to keep the fixtures small
BMM_CFGS = [(1, 1, 1, 1), (3, 5, 7, 9), (4, 33, 17, 65), (2, 64, 32, 48), (3, 130, 16, 24)]
ATTN_CFGS = [(2, 64, 16), (1, 100, 24), (1, 160, 32)]


def gen_bmm():
    out = {}
    R.set_seed(7)
    for (B, M, K, N) in BMM_CFGS:
        A, Bm = R.randn(B, M * K), R.randn(B, K * N)
        C = R.call("dream_bmm", A, Bm, *(R.scalar(v) for v in (B, M, K, N)))
        G = seeded_backward(C, (B, M * N))
        t = f"{B}_{M}_{K}_{N}"
        out[f"A_{t}"], out[f"B_{t}"], out[f"G_{t}"] = R.data(A), R.data(Bm), G
        out[f"C_{t}"], out[f"dA_{t}"], out[f"dB_{t}"] = R.data(C), R.grad(A), R.grad(Bm)
    np.savez_compressed(os.path.join(HERE, "bmm.npz"), **{k: v.astype(np.float32) for k, v in out.items()})


def gen_attn():
    out = {}
    R.set_seed(31)
    for causal in (0, 1):
        for (B, S, dk) in ATTN_CFGS:
            Q, K, V = R.randn(B, S * dk), R.randn(B, S * dk), R.randn(B, S * dk)
            O = R.call("dream_attention_causal" if causal else "dream_attention", Q, K, V,
                       *(R.scalar(v) for v in (B, S, dk)))
            G = seeded_backward(O, (B, S * dk))
            t = f"{causal}_{B}_{S}_{dk}"
            out[f"G_{t}"], out[f"O_{t}"] = G.reshape(B, S, dk), R.data(O).reshape(B, S, dk)
            for name, x in (("Q", Q), ("K", K), ("V", V)):
                out[f"{name}_{t}"] = R.data(x).reshape(B, S, dk)
                out[f"d{name}_{t}"] = R.grad(x).reshape(B, S, dk)
    np.savez_compressed(os.path.join(HERE, "attn.npz"), **{k: v.astype(np.float32) for k, v in out.items()})


# (N, Cin, H, W, Cout, KH, KW) for conv2d; plus (pad, stride) for the padded form
CONV_CFGS = [(2, 3, 8, 9, 4, 3, 3), (1, 2, 7, 5, 3, 2, 4), (3, 4, 10, 10, 8, 1, 1), (2, 5, 12, 11, 6, 5, 3)]
CONV_PAD_CFGS = [(2, 3, 8, 9, 4, 3, 3, 1, 1), (1, 2, 9, 7, 3, 3, 3, 1, 2), (2, 4, 11, 10, 5, 4, 2, 2, 3)]


def gen_conv():
    out = {}
    R.set_seed(13)
    for (N, Cin, H, W, Cout, KH, KW) in CONV_CFGS:
        X, K, b = R.randn(N, Cin * H * W), R.randn(Cout, Cin * KH * KW), R.randn(1, Cout)
        Y = R.call("dream_conv2d", X, K, b, *(R.scalar(v) for v in (H, W, KH, KW)))
        OH, OW = H - KH + 1, W - KW + 1
        G = seeded_backward(Y, (N, Cout * OH * OW))
        t = f"{N}_{Cin}_{H}_{W}_{Cout}_{KH}_{KW}"
        out[f"X_{t}"], out[f"K_{t}"], out[f"b_{t}"], out[f"G_{t}"] = R.data(X), R.data(K), R.data(b)[0], G
        out[f"Y_{t}"], out[f"dX_{t}"], out[f"dK_{t}"] = R.data(Y), R.grad(X), R.grad(K)
    for (N, Cin, H, W, Cout, KH, KW, pad, stride) in CONV_PAD_CFGS:
        X, K, b = R.randn(N, Cin * H * W), R.randn(Cout, Cin * KH * KW), R.randn(1, Cout)
        Y = R.call("dream_conv2d_padded", X, K, b, *(R.scalar(v) for v in (H, W, KH, KW, pad, stride)))
        t = f"p{N}_{Cin}_{H}_{W}_{Cout}_{KH}_{KW}_{pad}_{stride}"
        out[f"X_{t}"], out[f"K_{t}"], out[f"b_{t}"], out[f"Y_{t}"] = R.data(X), R.data(K), R.data(b)[0], R.data(Y)
    np.savez_compressed(os.path.join(HERE, "conv.npz"), **{k: v.astype(np.float32) for k, v in out.items()})


INT8_DIMS = [(48, 40), (24, 48), (10, 24)]  # (out, in) per layer


def _compiled_predict(c_path, func, X, workdir):
    """Outputs of an emitted predict function (compiled with cc) for the rows of X."""
    so = os.path.join(workdir, os.path.basename(c_path) + ".so")
    subprocess.run(["cc", "-O2", "-shared", "-fPIC", c_path, "-o", so, "-lm"], check=True)
    lib = C.CDLL(so)
    fn = getattr(lib, func)
    fn.argtypes = [C.c_void_p, C.c_void_p]
    fn.restype = None
    Y = []
    for x in np.ascontiguousarray(X, np.float32):
        y = np.zeros(INT8_DIMS[-1][0], np.float32)
        fn(x.ctypes.data, y.ctypes.data)
        Y.append(y)
    return np.stack(Y)


def gen_int8_export():
    from dreamcompiler_b200 import int8_export as IE
    R.set_seed(42)
    ck = R.call("dream_ckpt_new")
    layers = []
    for i, (o, n) in enumerate(INT8_DIMS):
        W, b = R.randn(o, n), R.randn(1, o)
        R.call("dream_ckpt_add", ck, R.call("dream_str_create", f"fc{i + 1}.weight".encode()), W)
        R.call("dream_ckpt_add", ck, R.call("dream_str_create", f"fc{i + 1}.bias".encode()), b)
        layers.append((f"fc{i + 1}", R.data(W), R.data(b)[0]))
    out_dir = os.path.join(HERE, "int8_export")
    os.makedirs(out_dir, exist_ok=True)
    X = np.random.default_rng(1).standard_normal((16, INT8_DIMS[0][1])).astype(np.float32)
    with tempfile.TemporaryDirectory(dir=HERE) as td:
        # relative prefix, so the emitted #include names the header alone
        cwd = os.getcwd()
        os.chdir(td)
        try:
            R.call("dream_export_c_header_int8", ck, R.call("dream_str_create", b"mlp_int8"),
                   R.call("dream_str_create", b"mlp_predict_int8"))
        finally:
            os.chdir(cwd)
        prefix = os.path.join(td, "mlp_int8")
        Y = _compiled_predict(prefix + ".c", "mlp_predict_int8", X, td)
        for ext in (".c", ".h"):
            shutil.copy(prefix + ext, os.path.join(out_dir, "mlp_int8" + ext))
        pc = os.path.join(td, "mlp_int8_pc")
        IE.export_c_header_int8_per_channel(layers, pc, "mlp_predict_int8_pc")
        Ypc = _compiled_predict(pc + ".c", "mlp_predict_int8_pc", X, td)
    arrays = {"X": X, "Y": Y, "Ypc": Ypc}
    for name, W, b in layers:
        arrays[f"{name}_W"], arrays[f"{name}_b"] = W, b
    np.savez_compressed(os.path.join(HERE, "int8_export.npz"), **arrays)


if __name__ == "__main__":
    # optional arguments name the fixtures to regenerate (default: all)
    gens = {"gemm": gen_gemm, "flash": gen_flash, "linear": gen_linear, "tp": gen_tp, "gpt": gen_gpt,
            "adamw": gen_adamw, "bmm": gen_bmm, "attn": gen_attn, "int8_export": gen_int8_export,
            "conv": gen_conv}
    for name in sys.argv[1:] or list(gens):
        gens[name]()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
