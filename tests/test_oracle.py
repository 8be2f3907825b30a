"""CPU: the oracle (oracle/dream_oracle.cpp) pinned against golden vectors
produced by the reference runtime itself (tests/golden/make_golden.py), plus
known-answer tests for the parts the reference does not export."""
import numpy as np
import pytest

from conftest import normwise

GEMM_SHAPES = [(1, 1, 1), (1, 7, 1), (5, 1, 9), (3, 4, 5), (7, 13, 17), (31, 33, 37), (64, 64, 64), (65, 63, 66),
               (128, 100, 96)]
FLASH_CFGS = [(64, 16, 8), (64, 16, 16), (128, 32, 32), (100, 24, 16), (128, 64, 64), (160, 64, 32)]


def test_rng_replays_reference_stream(orc, golden):
    """set_seed(42) + randn in the fixture's draw order (A, B, G per shape)
    reproduces the reference's std::mt19937/normal_distribution stream bit
    for bit (runtime/ops/elementwise.inc:30-55)."""
    g = golden("gemm")
    orc.set_seed(42)
    for (M, K, N) in GEMM_SHAPES:
        t = f"{M}x{K}x{N}"
        for name, shape in (("A", (M, K)), ("B", (K, N)), ("G", (M, N))):
            assert np.array_equal(orc.randn(*shape), g[f"{name}_{t}"]), (name, t)


@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_gemm_f64_and_backward(orc, golden, shape):
    g = golden("gemm")
    M, K, N = shape
    t = f"{M}x{K}x{N}"
    A, B, G = g[f"A_{t}"], g[f"B_{t}"], g[f"G_{t}"]
    assert normwise(orc.gemm_f64(A, B), g[f"C_{t}"]) < 1e-13
    dA, dB = orc.matmul_bwd(A, B, G)
    assert normwise(dA, g[f"dA_{t}"]) < 1e-13
    assert normwise(dB, g[f"dB_{t}"]) < 1e-13


@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_gemm_f32_mirror_path(orc, golden, shape):
    """The f32 path accumulates in fp32 (dream_gemm_f32); same arithmetic
    order per KC=256 block, so these short-K shapes agree to the last bits."""
    g = golden("gemm")
    M, K, N = shape
    t = f"{M}x{K}x{N}"
    C32 = orc.gemm_f32(g[f"A_{t}"].astype(np.float32), g[f"B_{t}"].astype(np.float32))
    assert normwise(C32, g[f"C32_{t}"]) < 1e-6


@pytest.mark.parametrize("cfg", FLASH_CFGS)
def test_flash_fwd_bwd(orc, golden, cfg):
    g = golden("flash")
    S, dk, Bc = cfg
    t = f"{S}_{dk}_{Bc}"
    Q, K, V, G = g[f"Q_{t}"], g[f"K_{t}"], g[f"V_{t}"], g[f"G_{t}"]
    O, lse = orc.flash_fwd(Q, K, V, Bc)
    assert normwise(O, g[f"O_{t}"]) < 1e-12
    # flash == materialised causal attention (flash_attention_selftest, rel < 1e-9)
    assert normwise(O, g[f"Ocausal_{t}"]) < 1e-9
    assert normwise(orc.attention(Q, K, V, causal=True), g[f"Ocausal_{t}"]) < 1e-12
    assert normwise(orc.attention(Q, K, V, causal=False), g[f"Ofull_{t}"]) < 1e-12
    dQ, dK, dV = orc.flash_bwd(Q, K, V, G)
    for name, x in (("dQ", dQ), ("dK", dK), ("dV", dV)):
        assert normwise(x, g[f"{name}_{t}"]) < 1e-11, name
    # LSE is consistent with O: log sum_j exp(s_ij) >= max_j s_ij
    s = np.einsum("bid,bjd->bij", Q, K) / np.sqrt(dk)
    s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
    ref_lse = np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1)) + s.max(-1)
    assert np.abs(lse - ref_lse).max() < 1e-10


def test_flash_backward_reference_test26(orc, golden):
    """tests/26_flash_backward.dream: set_seed(5), S=32, dk=16, block 8,
    backward(sum(o)) -> dO = 1."""
    g = golden("flash")
    Q, K, V = g["t26_Q"], g["t26_K"], g["t26_V"]
    O, _ = orc.flash_fwd(Q, K, V, 8)
    assert normwise(O, g["t26_O"]) < 1e-12
    dQ, dK, dV = orc.flash_bwd(Q, K, V, np.ones_like(O))
    assert normwise(dQ, g["t26_dQ"]) < 1e-11
    assert normwise(dK, g["t26_dK"]) < 1e-11
    assert normwise(dV, g["t26_dV"]) < 1e-11
    # the reference test's own pass condition, against materialised attention
    assert abs(np.abs(dQ).sum() - np.abs(g["t26_dQ"]).sum()) < 1e-7


@pytest.mark.parametrize("relu", [0, 1])
@pytest.mark.parametrize("dims", [(8, 16, 12), (33, 65, 17)])
def test_linear(orc, golden, relu, dims):
    g = golden("linear")
    t = f"{relu}_{dims[0]}_{dims[1]}_{dims[2]}"
    X, W, b, G = g[f"X_{t}"], g[f"W_{t}"], g[f"b_{t}"], g[f"G_{t}"]
    Y = orc.linear(X, W, b, relu=bool(relu))
    assert normwise(Y, g[f"Y_{t}"]) < 1e-13
    dX, dW, db = orc.linear_bwd(X, W, Y, G, relu=bool(relu))
    assert normwise(dX, g[f"dX_{t}"]) < 1e-13
    assert normwise(dW, g[f"dW_{t}"]) < 1e-13
    assert normwise(db, g[f"db_{t}"]) < 1e-13


@pytest.mark.parametrize("dims", [(12, 16, 24), (9, 10, 23)])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 5, 7])
def test_tp_matmul_column(orc, golden, dims, G):
    g = golden("tp")
    M, K, N = dims
    X, W = g[f"X_{M}_{K}_{N}"], g[f"W_{M}_{K}_{N}"]
    Y = orc.tp_matmul_column(X, W, G)
    # the reference self-test demands max_rel < 1e-12 against the un-split product
    assert normwise(Y, g[f"Y_{M}_{K}_{N}_{G}"]) < 1e-13
    widths = [orc.tp_shard(N, G, r)[1] for r in range(G)]
    assert sum(widths) == N and max(widths) - min(widths) <= 1
    assert widths == sorted(widths, reverse=True)  # the first N % G shards are the wide ones


def test_bf16_round_known_answers(orc):
    """dream_to_bf16 (runtime/nn/training.inc:1969-1976): round to nearest even."""
    ulp = 2.0 ** -7
    cases = {
        1.0: 1.0,
        1.0 + ulp / 2: 1.0,                 # tie -> even (1.0)
        1.0 + 1.5 * ulp: 1.0 + 2 * ulp,     # tie -> even mantissa
        1.0 + 0.75 * ulp: 1.0 + ulp,        # above half -> up
        -3.0 - ulp: -3.0,                   # below half ulp (ulp of 3 is 2^-6) -> down
        65504.0: 65536.0,
        0.0: 0.0,
        float("inf"): float("inf"),
    }
    x = np.array(list(cases.keys()), np.float32)
    out = orc.round_bf16(x)
    assert np.array_equal(out, np.array(list(cases.values()), np.float32))
    assert np.isnan(orc.round_bf16(np.array([np.nan], np.float32))[0])


def test_bf16_round_matches_torch(orc):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(200_000) * np.exp(rng.uniform(-20, 20, 200_000))).astype(np.float32)
    ours = orc.bf16_bits(x)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, t)


def test_int8_quantizer_known_answers(orc):
    """export_c_header_int8's per-tensor quantiser (training.inc:3668-3692)."""
    w = np.array([0.0, 1.27, -1.27, 0.005, 0.015, -0.635, 0.6350001], np.float64)
    q, scale = orc.quantize_per_tensor(w)
    assert scale == pytest.approx(0.01)
    assert q.tolist() == [0, 127, -127, 1, 2, -64, 64]   # lround: 0.5 -> 1, -63.5 -> -64 (half away from zero)
    q0, s0 = orc.quantize_per_tensor(np.zeros(5))
    assert s0 == 1.0 and not q0.any()


def test_dense_q_and_int_core(orc):
    rng = np.random.default_rng(1)
    B, N, K = 3, 17, 40
    X = rng.standard_normal((B, K)).astype(np.float32)
    W = rng.integers(-127, 128, (N, K)).astype(np.int8)
    sc = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    Y = orc.dense_q(X, W, sc, b)
    ref = b.astype(np.float64) + sc.astype(np.float64) * (X.astype(np.float64) @ W.astype(np.float64).T)
    assert normwise(Y, ref) < 1e-5
    Xq, sx = orc.quantize_rows(X)
    assert np.abs(Xq).max() <= 127
    assert np.allclose(sx, np.abs(X).max(1) / 127, rtol=1e-6)
    acc = orc.i8_gemm(Xq, W)
    assert np.array_equal(acc, Xq.astype(np.int64) @ W.astype(np.int64).T)


def test_gemm_rows_sampling(orc):
    rng = np.random.default_rng(2)
    A, B = rng.standard_normal((50, 30)), rng.standard_normal((30, 20))
    rows = np.array([0, 7, 49, 13], np.int32)
    assert normwise(orc.gemm_rows_f64(A, B, rows), (A @ B)[rows]) < 1e-14


BMM_CFGS = [(1, 1, 1, 1), (3, 5, 7, 9), (4, 33, 17, 65), (2, 64, 32, 48), (3, 130, 16, 24)]
ATTN_CFGS = [(2, 64, 16), (1, 100, 24), (1, 160, 32)]
F32_STORED = 1e-6  # the bmm / attn fixtures are stored as float32


@pytest.mark.parametrize("cfg", BMM_CFGS)
def test_bmm_and_backward(orc, golden, cfg):
    """dream_bmm and its "bmm" backward (reference runtime outputs)."""
    g = golden("bmm")
    B, M, K, N = cfg
    t = f"{B}_{M}_{K}_{N}"
    A, Bm, G = g[f"A_{t}"].reshape(B, M, K), g[f"B_{t}"].reshape(B, K, N), g[f"G_{t}"].reshape(B, M, N)
    assert normwise(orc.bmm(A, Bm), g[f"C_{t}"].reshape(B, M, N)) < F32_STORED
    dA, dB = orc.bmm_bwd(A, Bm, G)
    assert normwise(dA, g[f"dA_{t}"].reshape(B, M, K)) < F32_STORED
    assert normwise(dB, g[f"dB_{t}"].reshape(B, K, N)) < F32_STORED


@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("cfg", ATTN_CFGS)
def test_attention_and_backward(orc, golden, cfg, causal):
    """dream_attention / dream_attention_causal and their backward."""
    g = golden("attn")
    t = f"{causal}_{cfg[0]}_{cfg[1]}_{cfg[2]}"
    Q, K, V, G = (g[f"{n}_{t}"] for n in ("Q", "K", "V", "G"))
    assert normwise(orc.attention(Q, K, V, causal=bool(causal)), g[f"O_{t}"]) < F32_STORED
    dQ, dK, dV = orc.attention_bwd(Q, K, V, G, causal=bool(causal))
    for name, x in (("dQ", dQ), ("dK", dK), ("dV", dV)):
        assert normwise(x, g[f"{name}_{t}"]) < F32_STORED, name
    if causal:  # the causal backward equals the flash backward
        assert normwise(orc.flash_bwd(Q, K, V, G)[0], dQ) < 1e-9


CONV_CFGS = [(2, 3, 8, 9, 4, 3, 3), (1, 2, 7, 5, 3, 2, 4), (3, 4, 10, 10, 8, 1, 1), (2, 5, 12, 11, 6, 5, 3)]
CONV_PAD_CFGS = [(2, 3, 8, 9, 4, 3, 3, 1, 1), (1, 2, 9, 7, 3, 3, 3, 1, 2), (2, 4, 11, 10, 5, 4, 2, 2, 3)]


@pytest.mark.parametrize("cfg", CONV_CFGS)
def test_conv2d_and_backward(orc, golden, cfg):
    """dream_conv2d and its "conv2d" backward (reference runtime outputs)."""
    g = golden("conv")
    N, Cin, H, W, Cout, KH, KW = cfg
    t = "_".join(map(str, cfg))
    X = g[f"X_{t}"].reshape(N, Cin, H, W)
    K, b = g[f"K_{t}"], g[f"b_{t}"]
    OH, OW = orc.conv_out(H, W, KH, KW)
    G = g[f"G_{t}"].reshape(N, Cout, OH, OW)
    assert normwise(orc.conv2d_fwd(X, K, b, KH, KW), g[f"Y_{t}"].reshape(N, Cout, OH, OW)) < F32_STORED
    dX, dK = orc.conv2d_bwd(X, K, G, KH, KW)
    assert normwise(dX, g[f"dX_{t}"].reshape(X.shape)) < F32_STORED
    assert normwise(dK, g[f"dK_{t}"]) < F32_STORED


@pytest.mark.parametrize("cfg", CONV_PAD_CFGS)
def test_conv2d_padded(orc, golden, cfg):
    g = golden("conv")
    N, Cin, H, W, Cout, KH, KW, pad, stride = cfg
    t = "p" + "_".join(map(str, cfg))
    X = g[f"X_{t}"].reshape(N, Cin, H, W)
    OH, OW = orc.conv_out(H, W, KH, KW, pad, stride)
    Y = orc.conv2d_fwd(X, g[f"K_{t}"], g[f"b_{t}"], KH, KW, pad, stride)
    assert normwise(Y, g[f"Y_{t}"].reshape(N, Cout, OH, OW)) < F32_STORED


def test_conv2d_backward_is_the_gradient(orc):
    """With padding and stride (where the reference's backward reuses the
    unpadded geometry), the oracle's backward is checked by finite
    differences of its forward: <dY, conv(X + e*V)> - <dY, conv(X - e*V)>."""
    rng = np.random.default_rng(3)
    N, Cin, H, W, Cout, KH, KW, pad, stride = 2, 3, 7, 6, 4, 3, 2, 1, 2
    X = rng.standard_normal((N, Cin, H, W))
    K = rng.standard_normal((Cout, Cin * KH * KW))
    OH, OW = orc.conv_out(H, W, KH, KW, pad, stride)
    G = rng.standard_normal((N, Cout, OH, OW))
    dX, dK = orc.conv2d_bwd(X, K, G, KH, KW, pad, stride)
    VX, VK = rng.standard_normal(X.shape), rng.standard_normal(K.shape)
    e = 1e-6
    f = lambda x, k: float((orc.conv2d_fwd(x, k, None, KH, KW, pad, stride) * G).sum())
    assert abs((f(X + e * VX, K) - f(X - e * VX, K)) / (2 * e) - (dX * VX).sum()) < 1e-5 * abs((dX * VX).sum()) + 1e-6
    assert abs((f(X, K + e * VK) - f(X, K - e * VK)) / (2 * e) - (dK * VK).sum()) < 1e-5 * abs((dK * VK).sum()) + 1e-6
