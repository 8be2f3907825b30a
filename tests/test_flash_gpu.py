"""GPU parity of dgx_flash_fwd / dgx_flash_bwd against the oracle (the
reference's f64 online-softmax forward and 3-pass backward) on identical
seeded inputs rounded to bf16. Tolerance: normwise 1e-2 (bf16 operands, fp32
softmax statistics and accumulation); LSE absolute 1e-3."""
import math

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-2


def to_dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda", torch.bfloat16)


def host(x):
    return x.float().cpu().numpy().astype(np.float64)


def run(dgx, Q, K, V, dO, causal=True):
    q, k, v, do = (to_dev(x) for x in (Q, K, V, dO))
    O, L = dgx.flash_fwd(q, k, v, causal=causal)
    dQ, dK, dV = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
    dgx.sync_check()
    return host(O), L.cpu().numpy().astype(np.float64), host(dQ), host(dK), host(dV)


def check(orc, Q, K, V, dO, res):
    Qr, Kr, Vr, dOr = (orc.round_bf16(x).astype(np.float64) for x in (Q, K, V, dO))
    O, lse = orc.flash_fwd(Qr, Kr, Vr)
    dQ, dK, dV = orc.flash_bwd(Qr, Kr, Vr, dOr)
    o, l, dq, dk, dv = res
    assert normwise(o, O) < TOL
    assert np.abs(l - lse).max() < 1e-3
    assert normwise(dq, dQ) < TOL
    assert normwise(dk, dK) < TOL
    assert normwise(dv, dV) < TOL


@pytest.mark.parametrize("cfg", [(64, 16, 8), (64, 16, 16), (128, 32, 32), (100, 24, 16), (128, 64, 64),
                                 (160, 64, 32)])
def test_golden_configs(dgx, orc, golden, cfg):
    """flash_attention_selftest configs (training.inc:411) with the reference
    runtime's own inputs; G is the injected dO."""
    g = golden("flash")
    S, dk, Bc = cfg
    t = f"{S}_{dk}_{Bc}"
    Q, K, V, G = g[f"Q_{t}"], g[f"K_{t}"], g[f"V_{t}"], g[f"G_{t}"]
    res = run(dgx, Q, K, V, G)
    check(orc, Q, K, V, G, res)
    # and directly against the reference's f64 outputs on the unrounded inputs
    o, _, dq, dk_, dv = res
    assert normwise(o, g[f"O_{t}"]) < 2 * TOL
    assert normwise(dq, g[f"dQ_{t}"]) < 2 * TOL
    assert normwise(dk_, g[f"dK_{t}"]) < 2 * TOL
    assert normwise(dv, g[f"dV_{t}"]) < 2 * TOL


def test_reference_test26(dgx, orc, golden):
    g = golden("flash")
    Q, K, V = g["t26_Q"], g["t26_K"], g["t26_V"]
    res = run(dgx, Q, K, V, np.ones_like(Q))
    check(orc, Q, K, V, np.ones_like(Q), res)


@pytest.mark.parametrize("BH,S,D", [(2, 128, 64), (3, 384, 64), (2, 300, 64), (2, 1000, 64), (1, 1, 64),
                                    (2, 257, 32), (1, 129, 16), (2, 77, 20), (1, 200, 128), (4, 256, 8),
                                    (2, 256, 128), (3, 513, 128), (1, 300, 96), (2, 129, 80), (1, 1000, 128),
                                    (1, 64, 72), (2, 200, 136)])
@pytest.mark.parametrize("causal", [True, False])
def test_shapes(dgx, orc, BH, S, D, causal):
    """Ragged S, tensor-core head dims (8..128, multiples of 8; D > 64 takes
    the two-half tiles with P written over S) and the SIMT path (D=20, 136);
    causal and full attention."""
    orc.set_seed(1000 + BH * S + D)
    Q, K, V, dO = (orc.randn(BH, S, D) for _ in range(4))
    res = run(dgx, Q, K, V, dO, causal)
    Qr, Kr, Vr, dOr = (orc.round_bf16(x).astype(np.float64) for x in (Q, K, V, dO))
    if causal:
        check(orc, Q, K, V, dO, res)
    else:
        O = orc.attention(Qr, Kr, Vr, causal=False)
        assert normwise(res[0], O) < TOL
        # full-attention gradients via the materialised softmax
        s = np.einsum("bid,bjd->bij", Qr, Kr) / math.sqrt(D)
        P = np.exp(s - s.max(-1, keepdims=True))
        P /= P.sum(-1, keepdims=True)
        dV = np.einsum("bij,bid->bjd", P, dOr)
        dP = np.einsum("bid,bjd->bij", dOr, Vr)
        dS = P * (dP - (dP * P).sum(-1, keepdims=True))
        dQ = np.einsum("bij,bjd->bid", dS, Kr) / math.sqrt(D)
        dK = np.einsum("bij,bid->bjd", dS, Qr) / math.sqrt(D)
        assert normwise(res[2], dQ) < TOL
        assert normwise(res[3], dK) < TOL
        assert normwise(res[4], dV) < TOL


def test_config2_full_size(dgx, orc):
    """B=8, H=16, S=2048, D=64, bf16 Q/K/V/dO ~ N(0,1)
    (reference RNG, seed 42, order Q K V dO), scale 1/8. Eight heads, one in
    each batch entry and the last head among them, against the f64 oracle
    (O, LSE, dQ, dK, dV); every head through size-independent identities:
      row 0 of O is V_0 (causal), sum_j dV_j = sum_i dO_i (rows of P sum to 1),
      sum_j dK_j = 0 (rows of dS sum to 0)."""
    BH, S, D = 128, 2048, 64
    orc.set_seed(42)
    Q, K, V, dO = (orc.randn(BH, S, D) for _ in range(4))
    q, k, v, do = (to_dev(x) for x in (Q, K, V, dO))
    O, L = dgx.flash_fwd(q, k, v)
    dQ, dK, dV = dgx.flash_bwd(q, k, v, O, do, L)
    dgx.sync_check()
    hs = [0, 19, 37, 55, 73, 91, 109, 127]
    res = (host(O[hs]), L[hs].cpu().numpy().astype(np.float64), host(dQ[hs]), host(dK[hs]), host(dV[hs]))
    Qr, Kr, Vr, dOr = (orc.round_bf16(x[hs]).astype(np.float64) for x in (Q, K, V, dO))
    rO, rL = orc.flash_fwd(Qr, Kr, Vr)
    rdQ, rdK, rdV = orc.flash_bwd(Qr, Kr, Vr, dOr)
    for i, h in enumerate(hs):  # per head, so one bad head cannot hide under the others' scale
        o, l, dq, dk, dv = (r[i] for r in res)
        assert normwise(o, rO[i]) < TOL, h
        assert np.abs(l - rL[i]).max() < 1e-3, h
        assert normwise(dq, rdQ[i]) < TOL, h
        assert normwise(dk, rdK[i]) < TOL, h
        assert normwise(dv, rdV[i]) < TOL, h
    Of, vf, dof = O.float(), v.float(), do.float()
    assert (Of[:, 0] - vf[:, 0]).abs().max().item() < 1e-2
    colsum_dv = dV.float().sum(1)
    ref_dv = dof.sum(1)
    assert ((colsum_dv - ref_dv).abs().max() / ref_dv.abs().max()).item() < 2e-2
    colsum_dk = dK.float().sum(1).abs().max().item()
    assert colsum_dk / dK.float().abs().sum(1).max().item() < 2e-2
    assert torch.isfinite(dQ.float()).all() and torch.isfinite(L).all()


def test_d128_backward_is_reproducible(dgx):
    """For 64 < D <= 128 every gradient element has one owner (dK, dV per key
    tile, dQ per query tile): two runs give the same bits."""
    g = torch.Generator(device="cuda").manual_seed(8)
    q, k, v, do = (torch.randn(4, 700, 128, device="cuda", generator=g).bfloat16() for _ in range(4))
    O, L = dgx.flash_fwd(q, k, v)
    a = dgx.flash_bwd(q, k, v, O, do, L)
    b = dgx.flash_bwd(q, k, v, O, do, L)
    dgx.sync_check()
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("BH,S,D,causal", [(2, 384, 64, True), (3, 300, 64, True), (2, 257, 32, False),
                                           (1, 129, 16, True), (2, 1000, 64, False)])
def test_deterministic_mode(dgx, orc, BH, S, D, causal):
    """dgx_flash_set_deterministic(1): D <= 64 takes the two-kernel backward.
    It matches the oracle like the default path, gives the same bits on every
    run for dQ as well, and the same dK, dV bits as the default path (same
    per-element arithmetic, same accumulation order)."""
    orc.set_seed(500 + BH * S + D)
    Q, K, V, dO = (orc.randn(BH, S, D) for _ in range(4))
    q, k, v, do = (to_dev(x) for x in (Q, K, V, dO))
    O, L = dgx.flash_fwd(q, k, v, causal=causal)
    fast = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
    dgx.flash_set_deterministic(True)
    try:
        a = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
        b = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
    finally:
        dgx.flash_set_deterministic(False)
    dgx.sync_check()
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert torch.equal(a[1], fast[1]) and torch.equal(a[2], fast[2])
    if causal:
        check(orc, Q, K, V, dO, (host(O), L.cpu().numpy().astype(np.float64), host(a[0]), host(a[1]), host(a[2])))
    else:
        assert normwise(host(a[0]), host(fast[0])) < 1e-2


def test_workspace_contract(dgx):
    """Caller-supplied workspace: too small is rejected, exact size works."""
    BH, S, D = 2, 256, 64
    q, k, v, do = (torch.randn(BH, S, D, device="cuda").bfloat16() for _ in range(4))
    O, L = dgx.flash_fwd(q, k, v)
    need = dgx.flash_bwd_workspace_size(BH, S, D)
    small = torch.empty((need - 16) // 4, device="cuda")
    with pytest.raises(dgx.DgxError):
        dgx.flash_bwd(q, k, v, O, do, L, workspace=small)
    ws = torch.empty(need // 4, device="cuda")
    a = dgx.flash_bwd(q, k, v, O, do, L, workspace=ws)
    b = dgx.flash_bwd(q, k, v, O, do, L)
    dgx.sync_check()
    # dK, dV are written once per key tile: bit-identical. dQ is summed over
    # key tiles with fp32 atomics, so its last bits may differ between runs.
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    assert ((a[0].float() - b[0].float()).abs().max() / b[0].float().abs().max()).item() < 1e-2


@pytest.mark.parametrize("B,H,S,causal,D", [(2, 6, 256, True, 64), (1, 3, 300, True, 64), (2, 2, 200, False, 64),
                                            (1, 4, 128, True, 64), (2, 3, 384, True, 128), (1, 2, 200, False, 96)])
def test_head_rows_layout_matches_dense(dgx, B, H, S, causal, D):
    """dgx_flash_fwd_rows / dgx_flash_bwd_rows on heads inside token rows
    (a fused QKV buffer [B*S][3*H*D], O and dO [B*S][H*D]) give exactly the
    dense [BH][S][D] kernels' results on the same values (same tiles, same
    arithmetic: bit-identical)."""
    g = torch.Generator(device="cuda").manual_seed(B * 100 + H * 10 + S)
    qkv = torch.randn(B * S, 3 * H * D, device="cuda", generator=g).bfloat16()
    do_rows = torch.randn(B * S, H * D, device="cuda", generator=g).bfloat16()
    HD = H * D
    heads = lambda x: x.reshape(B, S, H, D).permute(0, 2, 1, 3).reshape(B * H, S, D).contiguous()
    rows = lambda x: x.reshape(B, H, S, D).permute(0, 2, 1, 3).reshape(B * S, HD)
    q, k, v, do = heads(qkv[:, :HD]), heads(qkv[:, HD:2 * HD]), heads(qkv[:, 2 * HD:]), heads(do_rows)
    O, L = dgx.flash_fwd(q, k, v, causal=causal)
    dQ, dK, dV = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
    o_rows = torch.empty(B * S, HD, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H, S, device="cuda")
    dgx.flash_fwd_rows(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], o_rows, lse, B, H, S, D, causal=causal)
    dqkv = torch.zeros(B * S, 3 * HD, device="cuda", dtype=torch.bfloat16)
    dgx.flash_bwd_rows(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], o_rows, do_rows, lse, dqkv[:, :HD],
                       dqkv[:, HD:2 * HD], dqkv[:, 2 * HD:], B, H, S, D, causal=causal)
    dgx.sync_check()
    assert torch.equal(o_rows, rows(O))
    assert torch.equal(lse, L)
    assert torch.equal(dqkv[:, :HD], rows(dQ))
    assert torch.equal(dqkv[:, HD:2 * HD], rows(dK))
    assert torch.equal(dqkv[:, 2 * HD:], rows(dV))


def test_head_rows_rejects_unsupported(dgx):
    x = torch.zeros(256, 3 * 2 * 40, device="cuda", dtype=torch.bfloat16)
    o = torch.zeros(256, 80, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(dgx.DgxError):  # D = 48 is fine, but O's pitch 80 < H*D = 96 is not
        dgx.flash_fwd_rows(x[:, :80], x[:, 80:160], x[:, 160:], o, torch.empty(2, 256, device="cuda"), 1, 2, 256, 48)


@pytest.mark.parametrize("BH,S,D,causal", [(8, 1024, 64, True), (3, 300, 32, False)])
def test_caller_workspace_cleared_behind_the_forward(dgx, BH, S, D, causal):
    """With a workspace of the caller's, the backward's row pre-pass clears the
    fp32 dQ accumulator in it before waiting for the kernel issued just before
    (here the forward). A workspace full of NaN before every step must give
    the dK, dV bits of the library-scratch path and its dQ up to the order of
    the fp32 reduce-adds, on back-to-back steps with alternating inputs."""
    g = torch.Generator(device="cuda").manual_seed(31 + S)
    sets = [[torch.randn(BH, S, D, device="cuda", generator=g).bfloat16() for _ in range(4)] for _ in range(2)]
    ws = torch.empty(dgx.flash_bwd_workspace_size(BH, S, D) // 4 + 1, device="cuda")
    for step in range(4):
        q, k, v, do = sets[step & 1]
        ws.fill_(float("nan"))
        O, L = dgx.flash_fwd(q, k, v, causal=causal)
        a = dgx.flash_bwd(q, k, v, O, do, L, causal=causal, workspace=ws)
        ref = dgx.flash_bwd(q, k, v, O, do, L, causal=causal)
        dgx.sync_check()
        assert torch.equal(a[1], ref[1]) and torch.equal(a[2], ref[2])
        assert torch.isfinite(a[0].float()).all()
        assert normwise(host(a[0]), host(ref[0])) < 1e-2
