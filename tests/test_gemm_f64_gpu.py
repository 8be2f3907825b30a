"""GPU: the f64 GEMM (dgx_gemm_f64) against the oracle's restatement of the
reference's f64 GEMM (dream_gemm_d, runtime/ops/elementwise.inc:516-638) and
its f64 "matmul" / "linear" backward (runtime/ops/autograd.inc:91-125,
:156-211). Both sides sum in f64, in different orders, so the gate is
normwise 1e-13 (a few ulps of the largest product sums)."""
import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-13


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float64)).cuda()


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (1, 1, 1), (129, 77, 300), (512, 2048, 64), (3000, 200, 513),
                                   (64, 64, 8), (2048, 2048, 16)])
def test_f64_against_oracle(dgx, orc, M, N, K):
    orc.set_seed(M + 3 * N + 7 * K)
    A, B = orc.randn(M, K), orc.randn(K, N)
    C = dgx.gemm(dev(A), dev(B))
    dgx.sync_check()
    assert C.dtype == torch.float64
    assert normwise(C.cpu().numpy(), orc.gemm_f64(A, B)) < TOL


def test_f64_config1_forward_backward(dgx, orc, golden):
    """BASELINE config 1 on f64 tensors (the reference's default dtype): the
    reference's own seeded A, B, dC; C = A.B, dA = dC.B^T, dB = A^T.dC
    accumulated into zero gradients (beta = 1)."""
    orc.set_seed(42)
    n = 1024
    A, B, dC = orc.randn(n, n), orc.randn(n, n), orc.randn(n, n)
    Ad, Bd, dCd = dev(A), dev(B), dev(dC)
    C = dgx.gemm(Ad, Bd)
    dA = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    dB = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    dgx.gemm(dCd, Bd, transB=True, out=dA, beta=1.0)
    dgx.gemm(Ad, dCd, transA=True, out=dB, beta=1.0)
    dgx.sync_check()
    rdA, rdB = orc.matmul_bwd(A, B, dC)
    assert normwise(C.cpu().numpy(), orc.gemm_f64(A, B)) < TOL
    assert normwise(dA.cpu().numpy(), rdA) < TOL
    assert normwise(dB.cpu().numpy(), rdB) < TOL


@pytest.mark.parametrize("transA,transB", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_f64_transposes_beta_bias_relu(dgx, orc, transA, transB):
    rng = np.random.default_rng(10 + 2 * transA + transB)
    M, N, K = 200, 130, 96
    A = rng.standard_normal((K, M) if transA else (M, K))
    B = rng.standard_normal((N, K) if transB else (K, N))
    C0 = rng.standard_normal((M, N))
    bias = rng.standard_normal(N)
    opA = A.T if transA else A
    opB = B.T if transB else B
    C = dev(C0)
    dgx.gemm(dev(A), dev(B), transA=bool(transA), transB=bool(transB), out=C, beta=0.5, bias=dev(bias), relu=True)
    dgx.sync_check()
    ref = np.maximum(0.5 * C0 + orc.gemm_f64(np.ascontiguousarray(opA), np.ascontiguousarray(opB)) + bias, 0)
    assert normwise(C.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("case", ["0_8_16_12", "0_33_65_17", "1_8_16_12", "1_33_65_17"])
def test_f64_linear_matches_reference_goldens(dgx, golden, case):
    """dream_linear[_relu] on f64 tensors, Y = X.W^T + b, and its backward
    dX = dY.W, dW = dY^T.X (dY masked by Y > 0 for the ReLU form), against the
    reference runtime's own outputs (tests/golden/linear.npz)."""
    g = golden("linear")
    X, W, b, G, Y = (g[f"{k}_{case}"] for k in ("X", "W", "b", "G", "Y"))
    relu = case.startswith("1")
    out = dgx.gemm(dev(X), dev(W), transB=True, bias=dev(b.ravel()), relu=relu)
    Gm = np.where(Y > 0, G, 0.0) if relu else G
    dX = dgx.gemm(dev(Gm), dev(W))
    dW = dgx.gemm(dev(Gm), dev(X), transA=True)
    dgx.sync_check()
    assert normwise(out.cpu().numpy(), Y) < TOL
    assert normwise(dX.cpu().numpy(), g[f"dX_{case}"]) < TOL
    assert normwise(dW.cpu().numpy(), g[f"dW_{case}"]) < TOL


def test_f64_pitched_operands(dgx, orc):
    rng = np.random.default_rng(4)
    big = rng.standard_normal((300, 400))
    Ab = dev(big)
    A = Ab[:, 7:7 + 250]          # pitch 400, odd start
    B = dev(rng.standard_normal((250, 90)))
    C = dgx.gemm(A, B)
    dgx.sync_check()
    assert normwise(C.cpu().numpy(), orc.gemm_f64(big[:, 7:257], B.cpu().numpy())) < TOL
