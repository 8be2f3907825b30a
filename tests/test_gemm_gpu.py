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
