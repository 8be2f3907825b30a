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


@pytest.mark.parametrize("B,N,K", [
    (3, 200, 48),       # one K block, ragged N, 3 plane rows padded to 16
    (33, 130, 4112),    # K % 128 != 0 (zero-filled tail), 2 output tiles, cluster split-K
    (100, 4096, 1024),  # W8A32: two activation chunks of 64 rows
    (300, 257, 256),    # W8A8: two chunks of 160 rows; W8A32: four of 80
    (17, 384, 8192),    # 8-way cluster split-K
    (2, 128, 20480),    # K beyond the register-resident pre-passes (looping forms)
    (40, 12804, 128),   # unsplit, TMA-stored output tiles, last tile 4 channels wide
])
def test_tensor_core_partitions(dgx, orc, B, N, K):
    """Shapes that exercise each way the tensor-core path divides the work:
    cluster split-K with the DSMEM reduction, activation chunks, tails."""
    X, W, sc, b = inputs(orc, B, N, K, seed=B * 7 + N + K)
    Xd, Wd, scd, bd = (torch.from_numpy(a).cuda() for a in (X, W, sc, b))
    Y0 = dgx.gemm_w8(Xd, Wd, scd, bd, mode=0)
    Y1 = dgx.gemm_w8(Xd, Wd, scd, bd, mode=1)
    Xq, sx = dgx.quantize_rows_i8(Xd)
    acc = dgx.gemm_i8i32(Xq, Wd)
    dgx.sync_check()
    assert normwise(Y0.cpu().numpy(), orc.dense_q(X, W, sc, b)) < 1e-5
    rXq, rsx = orc.quantize_rows(X)
    racc = orc.i8_gemm(rXq, W)
    assert np.array_equal(acc.cpu().numpy(), racc)
    ref1 = b.astype(np.float64) + sc.astype(np.float64) * rsx.astype(np.float64)[:, None] * racc
    assert normwise(Y1.cpu().numpy(), ref1) < 1e-6


def test_w8a32_extreme_rows(dgx, orc):
    """Rows spanning the fp32 range (tiny, huge, all-zero, a single spike):
    the power-of-two row scale keeps the plane split exact for each."""
    B, N, K = 6, 256, 512
    rng = np.random.default_rng(5)
    X = rng.standard_normal((B, K)).astype(np.float32)
    X[0] *= np.float32(1e-30)
    X[1] *= np.float32(1e30)
    X[2] = 0
    X[3] = 0
    X[3, 77] = -3.5
    X[4, ::2] = 0
    W = rng.integers(-128, 128, (N, K)).astype(np.int8)  # includes -128
    sc = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = np.zeros(N, np.float32)  # no bias: a 1e-29 output must stay visible
    Y = dgx.gemm_w8(*(torch.from_numpy(a).cuda() for a in (X, W, sc, b)), mode=0)
    dgx.sync_check()
    ref = sc.astype(np.float64) * (X.astype(np.float64) @ W.T.astype(np.float64))
    Yh = Y.cpu().numpy().astype(np.float64)
    for r in range(B):
        nr = np.linalg.norm(ref[r])
        if nr == 0:
            assert not Yh[r].any(), r
        else:
            assert np.linalg.norm(Yh[r] - ref[r]) / nr < 1e-5, r


@pytest.mark.parametrize("B,N,K", [
    (1, 4096, 4096),    # config 5, 4-CTA clusters
    (16, 4096, 4096),   # 16 rows
    (5, 384, 8192),     # 8-CTA clusters, 8 K blocks per CTA
    (11, 130, 4112),    # 7 CTAs per cluster, the last one 3 blocks with a 16-value tail
    (3, 1000, 1024),    # 8 CTAs of one block each
])
def test_w8a8_small_batches_exact(dgx, orc, B, N, K):
    """Small W8A8 batches (the split-K cluster form) against the oracle's
    quantiser and exact int32 products, rounded once in fp32: any activation
    quantised differently moves an output by scale*sx*|w| >> the 4-ulp bound
    used here. Rows include an all-zero row, a single spike, and values exactly
    halfway between two steps."""
    X, W, sc, b = inputs(orc, B, N, K, seed=B * 13 + N + K)
    if B >= 3:
        X[1] = 0
        X[2] = 0
        X[2, K // 3] = -2.75
    if B >= 5:
        # x = (j + 0.5) * sx exactly: ties, which round half away from zero
        step = np.float32(4.0) / np.float32(127.0)
        X[4] = 0
        X[4, 0] = 4.0
        X[4, 1:9] = (np.arange(8, dtype=np.float32) + np.float32(0.5)) * step * np.float32(np.where(np.arange(8) % 2, -1, 1))
    Xd, Wd, scd, bd = (torch.from_numpy(a).cuda() for a in (X, W, sc, b))
    Y = dgx.gemm_w8(Xd, Wd, scd, bd, mode=1)
    dgx.sync_check()
    rXq, rsx = orc.quantize_rows(X)
    racc = orc.i8_gemm(rXq, W).astype(np.float64)
    x = (sc[None, :] * rsx[:, None]).astype(np.float32).astype(np.float64)  # fp32 scale product, as the kernel
    ref = x * racc.astype(np.float32).astype(np.float64) + b.astype(np.float64)
    err = np.abs(Y.cpu().numpy().astype(np.float64) - ref)
    bound = 4 * 2.0 ** -23 * (np.abs(x * racc) + np.abs(b.astype(np.float64))) + 1e-30
    assert (err <= bound).all(), (np.argwhere(err > bound)[:5], err.max())
