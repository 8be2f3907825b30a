"""GPU parity of the int8 weight-only dense layer against
the oracle's restatement of the exported dense_q (training.inc:3738-3752):
W8A32 within 1e-5 normwise (fp32 accumulation order differs), W8A8 int32
accumulators bit-exact, activation quantisation bit-exact."""
import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def inputs(orc, B, N, K, seed=7):
    orc.set_seed(seed)
    X = orc.randn(B, K).astype(np.float32)
    W = np.clip(np.rint(orc.rand_uniform((N, K), -127.5, 127.5)), -127, 127).astype(np.int8)
    sc = orc.rand_uniform((N,), 1e-3, 1e-2).astype(np.float32)
    b = orc.randn(1, N)[0].astype(np.float32)
    return X, W, sc, b


@pytest.mark.parametrize("B", [1, 16, 256, 5])
def test_config5_shapes(dgx, orc, B):
    N = K = 4096
    X, W, sc, b = inputs(orc, B, N, K)
    Xd, Wd, scd, bd = (torch.from_numpy(a).cuda() for a in (X, W, sc, b))
    Y0 = dgx.gemm_w8(Xd, Wd, scd, bd, mode=0)
    Xq, sx = dgx.quantize_rows_i8(Xd)
    acc = dgx.gemm_i8i32(Xq, Wd)
    Y1 = dgx.gemm_w8(Xd, Wd, scd, bd, mode=1)
    dgx.sync_check()
    assert normwise(Y0.cpu().numpy(), orc.dense_q(X, W, sc, b)) < 1e-5
    rXq, rsx = orc.quantize_rows(X)
    assert np.array_equal(Xq.cpu().numpy(), rXq)
    assert np.array_equal(sx.cpu().numpy(), rsx)
    racc = orc.i8_gemm(rXq, W)
    assert np.array_equal(acc.cpu().numpy(), racc)            # bit-exact before the scale
    ref1 = b.astype(np.float64) + sc.astype(np.float64) * rsx.astype(np.float64)[:, None] * racc
    assert normwise(Y1.cpu().numpy(), ref1) < 1e-6


@pytest.mark.parametrize("B,N,K", [(3, 17, 40), (1, 1, 1), (2, 33, 4095), (7, 100, 513)])
def test_ragged(dgx, orc, B, N, K):
    X, W, sc, b = inputs(orc, B, N, K, seed=B + N + K)
    Xd, Wd, scd, bd = (torch.from_numpy(a).cuda() for a in (X, W, sc, b))
    Y0 = dgx.gemm_w8(Xd, Wd, scd, bd, mode=0)
    Xq, _ = dgx.quantize_rows_i8(Xd)
    acc = dgx.gemm_i8i32(Xq, Wd)
    dgx.sync_check()
    assert normwise(Y0.cpu().numpy(), orc.dense_q(X, W, sc, b)) < 1e-5
    assert np.array_equal(acc.cpu().numpy(), orc.i8_gemm(Xq.cpu().numpy(), W))


def test_per_tensor_export_semantics(dgx, orc):
    """The exporter's per-tensor quantiser feeding the per-channel kernel:
    scale[n] = the one tensor scale reproduces dense_q exactly in form."""
    rng = np.random.default_rng(3)
    Wf = rng.standard_normal((64, 128))
    q, s = orc.quantize_per_tensor(Wf)
    X = rng.standard_normal((4, 128)).astype(np.float32)
    sc = np.full(64, s, np.float32)
    b = rng.standard_normal(64).astype(np.float32)
    Y = dgx.gemm_w8(*(torch.from_numpy(a).cuda() for a in (X, q, sc, b)), mode=0)
    dgx.sync_check()
    assert normwise(Y.cpu().numpy(), orc.dense_q(X, q, sc, b)) < 1e-5
