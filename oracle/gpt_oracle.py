"""TEST INFRASTRUCTURE: f64 numpy restatement of the GPT training step of
BASELINE config 3, composed from the reference runtime's own ops the way a
Dream program composes them (compare examples/gpt/char_gpt.dream):

    x  = reshape(embedding(tok, W_tok), B, S*d) + reshape(P, 1, S*d)
    per layer:  h = layer_norm(x)
                x = x + sum_h linear(flash_attention(q_h, k_h, v_h), Wo_h) + bo
                x = x + linear(gelu(linear(layer_norm(x), W1, b1)), W2, b2)
    logits = linear(layer_norm(x), Wout, bout)
    loss   = nll_loss(log_softmax(logits), targets)

Each op follows the reference file it cites; backward follows
runtime/ops/autograd.inc. Used only by tests (checker), never by the product.
"""
from __future__ import annotations

import numpy as np

GELU_K = np.sqrt(2.0 / np.pi)


# ---------------------------------------------------------------- ops
def layer_norm(x):
    """runtime/io/builtins.inc:167-197: row-wise, no affine, eps 1e-5."""
    mu = x.mean(axis=1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
    inv = 1.0 / np.sqrt(var + 1e-5)
    return (x - mu) * inv, inv


def layer_norm_bwd(y, inv, dy):
    """runtime/ops/autograd.inc:453-470: dx = inv/C (C dy - sum dy - y sum(dy y))."""
    C = y.shape[1]
    return inv / C * (C * dy - dy.sum(axis=1, keepdims=True) - y * (dy * y).sum(axis=1, keepdims=True))


def gelu(x):
    """runtime/io/builtins.inc:548-560 (tanh form)."""
    return 0.5 * x * (1.0 + np.tanh(GELU_K * (x + 0.044715 * x ** 3)))


def gelu_bwd(x, dy):
    """runtime/ops/autograd.inc:293-303."""
    th = np.tanh(GELU_K * (x + 0.044715 * x ** 3))
    return (0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * GELU_K * (1.0 + 3 * 0.044715 * x * x)) * dy


def linear(x, W, b):
    """runtime/ops/elementwise.inc:1432-1521: Y = X W^T + b."""
    return x @ W.T + b


def log_softmax_nll(logits, target):
    """runtime/ops/elementwise.inc:1550-1603 (index targets) and their
    backward (runtime/ops/autograd.inc:212-245): loss and dlogits."""
    n = logits.shape[0]
    mx = logits.max(axis=1, keepdims=True)
    e = np.exp(logits - mx)
    s = e.sum(axis=1, keepdims=True)
    lp = logits - (mx + np.log(s))
    loss = -lp[np.arange(n), target].sum() / n
    d = e / s
    d[np.arange(n), target] -= 1.0
    return loss, d / n


def causal_attention(q, k, v):
    """Causal softmax(q k^T / sqrt(dk)) v per (batch*head): the function
    dream_flash_attention computes (runtime/nn/training.inc:284-401)."""
    S, dk = q.shape[-2], q.shape[-1]
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(dk)
    s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return p @ v, p


def causal_attention_bwd(q, k, v, p, do):
    """dV = P^T dO, dS = P (dP - rowsum(dP P)), dQ = dS K / sqrt(dk),
    dK = dS^T Q / sqrt(dk) (runtime/ops/autograd.inc:779-840)."""
    sc = 1.0 / np.sqrt(q.shape[-1])
    dv = np.swapaxes(p, -1, -2) @ do
    dp = do @ np.swapaxes(v, -1, -2)
    ds = p * (dp - (dp * p).sum(axis=-1, keepdims=True))
    return ds @ k * sc, np.swapaxes(ds, -1, -2) @ q * sc, dv


def adamw(p, g, m, v, step, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.01):
    """runtime/io/builtins.inc:578-617 (one step, returns new p, m, v)."""
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    mh = m / (1 - b1 ** step)
    vh = v / (1 - b2 ** step)
    return p - lr * (mh / (np.sqrt(vh) + eps) + wd * p), m, v


# ---------------------------------------------------------------- model
def param_shapes(L, d, V, S):
    """Parameter names and shapes (W [out][in], the reference convention)."""
    shapes = {"W_tok": (V, d), "P": (S, d)}
    for l in range(L):
        shapes.update({f"Wqkv{l}": (3 * d, d), f"bqkv{l}": (3 * d,), f"Wo{l}": (d, d), f"bo{l}": (d,),
                       f"W1{l}": (4 * d, d), f"b1{l}": (4 * d,), f"W2{l}": (d, 4 * d), f"b2{l}": (d,)})
    shapes.update({"Wout": (V, d), "bout": (V,)})
    return shapes


def init_params(L, d, V, S, seed):
    """Seeded N(0, 0.02) weights (scaled down in the residual outputs), zero
    biases except small random ones so their gradients are exercised."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shp in param_shapes(L, d, V, S).items():
        std = 0.02 if name[0] in "WP" else 0.01
        if name.startswith(("Wo", "W2")):
            std = 0.02 / np.sqrt(2 * L)
        out[name] = (rng.standard_normal(shp) * std).astype(np.float32)
    return out


def step(params, tok, tgt, L, d, H, B, S, V):
    """Forward + backward of one step in f64: returns (loss, grads)."""
    P = {k: v.astype(np.float64) for k, v in params.items()}
    hd = d // H
    n = B * S
    x = P["W_tok"][tok] + np.tile(P["P"], (B, 1))
    cache = []
    for l in range(L):
        h, inv1 = layer_norm(x)
        qkv = linear(h, P[f"Wqkv{l}"], P[f"bqkv{l}"])
        heads = lambda t: t.reshape(B, S, H, hd).transpose(0, 2, 1, 3)
        q, k, v = (heads(qkv[:, i * d:(i + 1) * d]) for i in range(3))
        o, p = causal_attention(q, k, v)
        att = o.transpose(0, 2, 1, 3).reshape(n, d)
        x1 = x + linear(att, P[f"Wo{l}"], P[f"bo{l}"])
        h2, inv2 = layer_norm(x1)
        u = linear(h2, P[f"W1{l}"], P[f"b1{l}"])
        g = gelu(u)
        x2 = x1 + linear(g, P[f"W2{l}"], P[f"b2{l}"])
        cache.append((h, inv1, q, k, v, p, att, h2, inv2, u, g))
        x = x2
    hf, invf = layer_norm(x)
    logits = linear(hf, P["Wout"], P["bout"])
    loss, dlog = log_softmax_nll(logits, tgt)

    G = {}
    G["Wout"] = dlog.T @ hf
    G["bout"] = dlog.sum(0)
    dx = layer_norm_bwd(hf, invf, dlog @ P["Wout"])
    for l in reversed(range(L)):
        h, inv1, q, k, v, p, att, h2, inv2, u, g = cache[l]
        G[f"W2{l}"] = dx.T @ g
        G[f"b2{l}"] = dx.sum(0)
        du = gelu_bwd(u, dx @ P[f"W2{l}"])
        G[f"W1{l}"] = du.T @ h2
        G[f"b1{l}"] = du.sum(0)
        dx = dx + layer_norm_bwd(h2, inv2, du @ P[f"W1{l}"])
        G[f"Wo{l}"] = dx.T @ att
        G[f"bo{l}"] = dx.sum(0)
        datt = (dx @ P[f"Wo{l}"]).reshape(B, S, H, hd).transpose(0, 2, 1, 3)
        dq, dk, dv = causal_attention_bwd(q, k, v, p, datt)
        rows = lambda t: t.transpose(0, 2, 1, 3).reshape(n, d)
        dqkv = np.concatenate([rows(dq), rows(dk), rows(dv)], axis=1)
        G[f"Wqkv{l}"] = dqkv.T @ h
        G[f"bqkv{l}"] = dqkv.sum(0)
        dx = dx + layer_norm_bwd(h, inv1, dqkv @ P[f"Wqkv{l}"])
    G["W_tok"] = np.zeros_like(P["W_tok"])
    np.add.at(G["W_tok"], tok, dx)
    G["P"] = dx.reshape(B, S, d).sum(0)
    return loss, G
