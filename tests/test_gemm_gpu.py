"""GPU parity of dgx_gemm against the oracle (f64 GEMM on identical seeded
inputs) and the reference's golden vectors. Tolerances (normwise,
max|d|/max|ref|): f32 inputs 1e-4, bf16 inputs 1e-2 against the f64 product
of the bf16-rounded inputs."""
import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F32_TOL, BF16_TOL = 1e-4, 1e-2
GEMM_SHAPES = [(1, 1, 1), (1, 7, 1), (5, 1, 9), (3, 4, 5), (7, 13, 17), (31, 33, 37), (64, 64, 64), (65, 63, 66),
               (128, 100, 96)]


def cuda(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def bf16_round(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).bfloat16().float().numpy().astype(np.float64)


@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_golden_shapes_forward_and_backward(dgx, golden, shape):
    """gemm_selftest's shapes through the f32 path: C = A@B, dA = G.B^T, dB = A^T.G
    against the reference runtime's own tensor_matmul / "matmul" backward."""
    g = golden("gemm")
    M, K, N = shape
    t = f"{M}x{K}x{N}"
    A, B, G = cuda(g[f"A_{t}"]), cuda(g[f"B_{t}"]), cuda(g[f"G_{t}"])
    C = dgx.gemm(A, B)
    dA = torch.zeros(M, K, device="cuda")
    dB = torch.zeros(K, N, device="cuda")
    dgx.gemm(G, B, transB=True, out=dA, beta=1.0)
    dgx.gemm(A, G, transA=True, out=dB, beta=1.0)
    dgx.sync_check()
    assert normwise(C.cpu().numpy(), g[f"C_{t}"]) < F32_TOL
    assert normwise(C.cpu().numpy(), g[f"C32_{t}"]) < F32_TOL
    assert normwise(dA.cpu().numpy(), g[f"dA_{t}"]) < F32_TOL
    assert normwise(dB.cpu().numpy(), g[f"dB_{t}"]) < F32_TOL


def test_config1_f32_1024_forward_backward(dgx, orc):
    """set_seed(42); A, B, dC = randn(1024,1024) (reference
    RNG order); C = A@B and dA = dC.B^T, dB = A^T.dC against the f64 oracle."""
    n = 1024
    orc.set_seed(42)
    A, B, dC = orc.randn(n, n), orc.randn(n, n), orc.randn(n, n)
    Ad, Bd, dCd = cuda(A), cuda(B), cuda(dC)
    C = dgx.gemm(Ad, Bd)
    dA = dgx.gemm(dCd, Bd, transB=True)
    dB = dgx.gemm(Ad, dCd, transA=True)
    dgx.sync_check()
    A32, B32, dC32 = (x.astype(np.float32).astype(np.float64) for x in (A, B, dC))
    assert normwise(C.cpu().numpy(), orc.gemm_f64(A32, B32)) < F32_TOL
    rdA, rdB = orc.matmul_bwd(A32, B32, dC32)
    assert normwise(dA.cpu().numpy(), rdA) < F32_TOL
    assert normwise(dB.cpu().numpy(), rdB) < F32_TOL
    # the reference's own f32 path (fp32 accumulation) agrees at the same level
    assert normwise(C.cpu().numpy(), orc.gemm_f32(A, B)) < F32_TOL
    # FFMA mode, same contract
    C2 = dgx.gemm(Ad, Bd, f32_mode=1)
    dgx.sync_check()
    assert normwise(C2.cpu().numpy(), orc.gemm_f64(A32, B32)) < F32_TOL


@pytest.mark.parametrize("tA", [0, 1])
@pytest.mark.parametrize("tB", [0, 1])
@pytest.mark.parametrize("shape", [(256, 512, 128), (300, 200, 257), (129, 257, 136), (1, 8, 64), (8, 1, 8)])
def test_bf16_transposes_ragged(dgx, orc, tA, tB, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((K, M) if tA else (M, K))
    B = rng.standard_normal((N, K) if tB else (K, N))
    C = dgx.gemm(cuda(A, torch.bfloat16), cuda(B, torch.bfloat16), transA=bool(tA), transB=bool(tB))
    dgx.sync_check()
    Ar, Br = bf16_round(A), bf16_round(B)
    ref = orc.gemm_f64(Ar.T.copy() if tA else Ar, Br.T.copy() if tB else Br)
    assert normwise(C.cpu().numpy(), ref) < BF16_TOL


@pytest.mark.parametrize("tA", [0, 1])
@pytest.mark.parametrize("tB", [0, 1])
@pytest.mark.parametrize("shape", [(128, 256, 64), (300, 200, 257), (77, 33, 5)])
def test_f32_transposes_ragged(dgx, orc, tA, tB, shape):
    M, N, K = shape
    rng = np.random.default_rng(M + N * 3 + K)
    A = rng.standard_normal((K, M) if tA else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tB else (K, N)).astype(np.float32)
    C = dgx.gemm(cuda(A), cuda(B), transA=bool(tA), transB=bool(tB))
    dgx.sync_check()
    ref = orc.gemm_f64(A.T.astype(np.float64).copy() if tA else A.astype(np.float64),
                       B.T.astype(np.float64).copy() if tB else B.astype(np.float64))
    assert normwise(C.cpu().numpy(), ref) < F32_TOL


def test_linear_epilogues_against_reference(dgx, golden, orc):
    """dream_linear / dream_linear_relu: Y = X.W^T + b (+ReLU) in the epilogue."""
    g = golden("linear")
    for relu in (0, 1):
        for dims in [(8, 16, 12), (33, 65, 17)]:
            t = f"{relu}_{dims[0]}_{dims[1]}_{dims[2]}"
            X, W, b = cuda(g[f"X_{t}"]), cuda(g[f"W_{t}"]), cuda(g[f"b_{t}"])
            Y = dgx.gemm(X, W, transB=True, bias=b, relu=bool(relu))
            dgx.sync_check()
            assert normwise(Y.cpu().numpy(), g[f"Y_{t}"]) < F32_TOL


def test_beta_accumulate_and_bf16_output(dgx, orc):
    rng = np.random.default_rng(5)
    A = rng.standard_normal((256, 192)).astype(np.float32)
    B = rng.standard_normal((192, 320)).astype(np.float32)
    C0 = rng.standard_normal((256, 320)).astype(np.float32)
    Cd = cuda(C0)
    dgx.gemm(cuda(A), cuda(B), out=Cd, beta=1.0)
    dgx.sync_check()
    ref = C0.astype(np.float64) + orc.gemm_f64(A.astype(np.float64), B.astype(np.float64))
    assert normwise(Cd.cpu().numpy(), ref) < F32_TOL
    Cb = dgx.gemm(cuda(A, torch.bfloat16), cuda(B, torch.bfloat16), out_dtype=torch.bfloat16)
    dgx.sync_check()
    assert normwise(Cb.float().cpu().numpy(), orc.gemm_f64(bf16_round(A), bf16_round(B))) < BF16_TOL


def test_unaligned_pitch_uses_simt_path(dgx, orc):
    """A row pitch that TMA cannot describe (not a multiple of 16 bytes) still
    computes correctly on the device (SIMT kernel)."""
    rng = np.random.default_rng(6)
    big = cuda(rng.standard_normal((100, 67)), torch.bfloat16)
    A = big[:, :61]  # pitch 67 bf16 = 134 bytes
    B = cuda(rng.standard_normal((61, 40)), torch.bfloat16)
    C = dgx.gemm(A, B)
    dgx.sync_check()
    ref = orc.gemm_f64(A.float().cpu().numpy().astype(np.float64), B.float().cpu().numpy().astype(np.float64))
    assert normwise(C.cpu().numpy(), ref) < BF16_TOL


def test_degenerate_sizes(dgx):
    A = torch.zeros(0, 8, device="cuda")
    B = torch.ones(8, 4, device="cuda")
    assert dgx.gemm(A, B).shape == (0, 4)
    # K = 0: C = beta*C + bias
    A0, B0 = torch.zeros(3, 0, device="cuda"), torch.zeros(0, 5, device="cuda")
    bias = torch.arange(5, device="cuda", dtype=torch.float32)
    C = dgx.gemm(A0, B0, bias=bias)
    dgx.sync_check()
    assert torch.equal(C.cpu(), bias.cpu().expand(3, 5))


def test_known_answer_ones(dgx):
    """tests/09_matmul.dream and tests/10_f32_matmul.dream: ones(2,3)@ones(3,2) = 3,
    sum(ones(2,2)@ones(2,2)) = 8."""
    C = dgx.gemm(torch.ones(2, 3, device="cuda"), torch.ones(3, 2, device="cuda"))
    assert torch.equal(C.cpu(), torch.full((2, 2), 3.0))
    C = dgx.gemm(torch.ones(2, 2, device="cuda", dtype=torch.bfloat16), torch.ones(2, 2, device="cuda",
                                                                                   dtype=torch.bfloat16))
    assert C.sum().item() == 8.0


def test_config4_bf16_4096_full_and_16384_sampled(dgx, orc):
    """BASELINE config 4 shapes: A, B ~ N(0,1)/sqrt(K) (reference RNG), RNE to
    bf16, fp32 accumulate. 4096^3 checked in full; 16384^3 on 256 sampled rows."""
    for n, rows in ((4096, None), (16384, 256)):
        orc.set_seed(42)
        A = orc.randn(n, n) / np.sqrt(n)
        B = orc.randn(n, n) / np.sqrt(n)
        Ab, Bb = orc.round_bf16(A).astype(np.float64), orc.round_bf16(B).astype(np.float64)
        C = dgx.gemm(cuda(A, torch.bfloat16), cuda(B, torch.bfloat16))
        dgx.sync_check()
        Cn = C.cpu().numpy()
        if rows is None:
            ref = orc.gemm_f64(Ab, Bb)
            assert normwise(Cn, ref) < BF16_TOL
        else:
            idx = np.random.default_rng(0).choice(n, rows, replace=False).astype(np.int32)
            ref = orc.gemm_rows_f64(Ab, Bb, idx)
            assert normwise(Cn[idx], ref) < BF16_TOL
        del A, B, Ab, Bb, C


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("shape,tA", [((384, 384, 16384), 1), ((200, 130, 8192), 0), ((72, 384, 4096), 1)])
def test_split_k_small_outputs_long_k(dgx, orc, dtype, shape, tA):
    """Small outputs over a long K (the weight-gradient GEMMs dW = dY^T X)
    take the split-K path: K slices on separate CTAs, fp32 partial tiles
    summed in a fixed order, then the bias / beta / ReLU epilogue."""
    M, N, K = shape
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((K, M) if tA else (M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    td = torch.bfloat16 if dtype == "bf16" else torch.float32
    Ad, Bd = cuda(A, td), cuda(B, td)
    Ar = bf16_round(A) if dtype == "bf16" else A.astype(np.float64)
    Br = bf16_round(B) if dtype == "bf16" else B.astype(np.float64)
    ref = (Ar.T if tA else Ar) @ Br
    tol = BF16_TOL if dtype == "bf16" else F32_TOL
    C = dgx.gemm(Ad, Bd, transA=bool(tA))
    Cb = cuda(C0)
    dgx.gemm(Ad, Bd, transA=bool(tA), out=Cb, beta=1.0, bias=cuda(bias), relu=True)
    C16 = dgx.gemm(Ad, Bd, transA=bool(tA), out_dtype=torch.bfloat16)
    dgx.sync_check()
    assert normwise(C.cpu().numpy(), ref) < tol
    assert normwise(Cb.cpu().numpy(), np.maximum(ref + C0 + bias, 0)) < tol
    assert normwise(C16.float().cpu().numpy(), ref) < max(tol, 1e-2)
    # deterministic: the same call twice gives the same bits
    C2 = dgx.gemm(Ad, Bd, transA=bool(tA))
    dgx.sync_check()
    assert torch.equal(C, C2)


@pytest.mark.parametrize("algo", [0, 1])
@pytest.mark.parametrize("shape,tB,cdt,beta,bias,relu", [
    ((512, 768, 1024), True, "f32", 0.0, True, False),
    ((1000, 600, 1100), False, "f32", 1.0, True, False),      # ragged M, N, K; fp32 accumulate
    ((2048, 1152, 1536), True, "bf16", 0.0, True, True),
    ((8448, 8192, 1024), False, "bf16", 0.0, False, False),  # many 256 x 256 pair tiles
])
def test_two_sm_and_single_cta_kernels_agree(dgx, algo, shape, tB, cdt, beta, bias, relu):
    """The bf16 GEMM through the single-CTA kernel (algo 0) and through the
    2-SM CTA-pair kernel (algo 1, tcgen05 cta_group::2) against the f64
    product of the same bf16 inputs."""
    from dreamcompiler_b200 import _lib
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K + algo)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn((N, K) if tB else (K, N), device="cuda", generator=g).bfloat16()
    td = torch.float32 if cdt == "f32" else torch.bfloat16
    C0 = torch.randn(M, N, device="cuda", generator=g).to(td)
    bb = torch.randn(N, device="cuda", generator=g) if bias else None
    C = C0.clone()
    try:
        _lib.call("dgx_gemm_set_algo", algo)
        dgx.gemm(A, B, transB=tB, out=C, beta=beta, bias=bb, relu=relu)
        dgx.sync_check()
    finally:
        _lib.call("dgx_gemm_set_algo", 1)
    ref = A.double() @ (B.double().t() if tB else B.double())
    if beta:
        ref += C0.double()
    if bias:
        ref += bb.double()
    if relu:
        ref = ref.clamp_min(0)
    assert normwise(C.double().cpu().numpy(), ref.cpu().numpy()) < (1e-5 if cdt == "f32" else 1e-2)


BMM_CFGS = [(1, 1, 1, 1), (3, 5, 7, 9), (4, 33, 17, 65), (2, 64, 32, 48), (3, 130, 16, 24)]


@pytest.mark.parametrize("cfg", BMM_CFGS)
def test_bmm_golden(dgx, orc, golden, cfg):
    """dream_bmm's own outputs and "bmm" backward (reference runtime) through
    dgx_bmm / dgx_gemm_batched: f32 (3xTF32) and bf16 operands."""
    g = golden("bmm")
    B, M, K, N = cfg
    t = f"{B}_{M}_{K}_{N}"
    A, Bm, G = (g[f"{n}_{t}"].reshape(s) for n, s in (("A", (B, M, K)), ("B", (B, K, N)), ("G", (B, M, N))))
    Ad, Bd, Gd = cuda(A), cuda(Bm), cuda(G)
    C = dgx.bmm(Ad, Bd)
    dA = dgx.gemm_batched(Gd, Bd, transB=True)
    dB = dgx.gemm_batched(Ad, Gd, transA=True)
    dgx.sync_check()
    assert normwise(C.cpu().numpy(), g[f"C_{t}"].reshape(B, M, N)) < F32_TOL
    assert normwise(dA.cpu().numpy(), g[f"dA_{t}"].reshape(B, M, K)) < F32_TOL
    assert normwise(dB.cpu().numpy(), g[f"dB_{t}"].reshape(B, K, N)) < F32_TOL
    Cb = dgx.bmm(Ad.bfloat16(), Bd.bfloat16())
    dgx.sync_check()
    assert normwise(Cb.cpu().numpy(), orc.bmm(bf16_round(A), bf16_round(Bm))) < BF16_TOL


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("batch,M,N,K,ta,tb", [(5, 200, 136, 72, 0, 0), (3, 130, 264, 520, 1, 0),
                                               (7, 96, 40, 1100, 0, 1), (2, 257, 300, 64, 1, 1),
                                               (4, 33, 65, 17, 0, 0), (9, 128, 128, 128, 0, 0)])
def test_gemm_batched_shapes(dgx, orc, dtype, batch, M, N, K, ta, tb):
    """One launch over all batches: ragged tiles at every batch boundary,
    transposed operands, beta=1 accumulation; K=17 (bf16) takes the SIMT
    path. Each batch against the f64 oracle."""
    rng = np.random.default_rng(batch * 1000 + M + N + K)
    A = rng.standard_normal((batch, K, M) if ta else (batch, M, K))
    B = rng.standard_normal((batch, N, K) if tb else (batch, K, N))
    C0 = rng.standard_normal((batch, M, N))
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    Ad, Bd = cuda(A, tdt), cuda(B, tdt)
    out = cuda(C0)
    dgx.gemm_batched(Ad, Bd, transA=bool(ta), transB=bool(tb), out=out, beta=1.0)
    dgx.sync_check()
    Ar, Br = (x if dtype == "f32" else bf16_round(x) for x in (A, B))
    if ta:
        Ar = Ar.transpose(0, 2, 1)
    if tb:
        Br = Br.transpose(0, 2, 1)
    ref = orc.bmm(Ar, Br) + C0
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    got = out.cpu().numpy()
    for b in range(batch):
        assert normwise(got[b], ref[b]) < tol, b


def test_bmm_many_batches_and_strided_views(dgx, orc):
    """More batches than one launch's grid z extent (33000 > 32767: two
    launches), and batch / row strides that are not the dense ones (views
    into wider buffers)."""
    rng = np.random.default_rng(5)
    A, B = rng.standard_normal((33000, 2, 4)), rng.standard_normal((33000, 4, 8))
    C = dgx.bmm(cuda(A), cuda(B))
    dgx.sync_check()
    assert normwise(C.cpu().numpy(), np.einsum("bmk,bkn->bmn", A, B)) < F32_TOL
    big = torch.randn(6, 80, 96, device="cuda").bfloat16()
    Bw = torch.randn(6, 64, 72, device="cuda").bfloat16()
    Av, Bv = big[:, 8:72, 16:80], Bw[:, :, :40]  # [6, 64, 64] x [6, 64, 40], padded pitches
    out = torch.zeros(6, 64, 48, device="cuda")[:, :, :40]
    dgx.gemm_batched(Av, Bv, out=out)
    dgx.sync_check()
    ref = np.einsum("bmk,bkn->bmn", Av.double().cpu().numpy(), Bv.double().cpu().numpy())
    assert normwise(out.cpu().numpy(), ref) < BF16_TOL


def test_bmm_broadcast_operand_and_overlap_rejected(dgx):
    """Batch stride 0 shares one operand across batches; overlapping output
    batches are rejected with DGX_EINVAL."""
    W = torch.randn(1, 48, 40, device="cuda")
    X = torch.randn(5, 24, 48, device="cuda")
    out = dgx.gemm_batched(X, W.expand(5, 48, 40))
    dgx.sync_check()
    ref = np.einsum("bmk,kn->bmn", X.double().cpu().numpy(), W[0].double().cpu().numpy())
    assert normwise(out.cpu().numpy(), ref) < F32_TOL
    A = torch.zeros(2, 4, 4, device="cuda")
    with pytest.raises(dgx.DgxError):
        dgx.gemm_batched(A, A, out=torch.zeros(1, 4, 4, device="cuda").expand(2, 4, 4))


@pytest.mark.parametrize("M,K,N", [(256, 128, 256), (300, 200, 257), (512, 64, 300), (8, 16, 16), (7, 15, 13),
                                   (9, 8, 17), (1, 4, 1), (16, 32, 24), (32, 16, 32)])
def test_reference_selftest_shapes(dgx, orc, M, K, N):
    """The shapes of the reference's gpu_selftest (runtime/ops/elementwise.inc:
    821: the GPU matmul against the CPU GEMM, uniform(-1, 1) inputs, pass at
    |d| <= sqrt(K)*1e-4 elementwise) and of its packed-f32 check (:939-941),
    on the 3xTF32 path: the reference's elementwise criterion and the
    normwise 1e-4 gate both hold."""
    rng = np.random.default_rng(20260708 + M + K + N)
    A = rng.uniform(-1, 1, (M, K))
    B = rng.uniform(-1, 1, (K, N))
    C = dgx.gemm(cuda(A), cuda(B))
    dgx.sync_check()
    ref = orc.gemm_f64(A.astype(np.float32).astype(np.float64), B.astype(np.float32).astype(np.float64))
    got = C.cpu().numpy().astype(np.float64)
    assert np.abs(got - ref).max() <= np.sqrt(K) * 1e-4
    assert normwise(got, ref) < F32_TOL
