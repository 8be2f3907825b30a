"""GPU parity of dgx_conv2d_fwd / dgx_conv2d_bwd (im2col + one tensor-core
GEMM per pass) against the reference runtime's conv2d outputs and the f64
oracle. Tolerances (normwise): fp32 operands (3xTF32) 1e-4; bf16 operands
2e-2 against the f64 result on the unrounded inputs."""
import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F32_TOL, BF16_TOL = 1e-4, 2e-2
CONV_CFGS = [(2, 3, 8, 9, 4, 3, 3), (1, 2, 7, 5, 3, 2, 4), (3, 4, 10, 10, 8, 1, 1), (2, 5, 12, 11, 6, 5, 3)]
CONV_PAD_CFGS = [(2, 3, 8, 9, 4, 3, 3, 1, 1), (1, 2, 9, 7, 3, 3, 3, 1, 2), (2, 4, 11, 10, 5, 4, 2, 2, 3)]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("operands", ["f32", "bf16"])
@pytest.mark.parametrize("cfg", CONV_CFGS)
def test_reference_conv2d(dgx, golden, cfg, operands):
    g = golden("conv")
    N, Cin, H, W, Cout, KH, KW = cfg
    t = "_".join(map(str, cfg))
    OH, OW = H - KH + 1, W - KW + 1
    X, K, b = cuda(g[f"X_{t}"].reshape(N, Cin, H, W)), cuda(g[f"K_{t}"]), cuda(g[f"b_{t}"])
    G = cuda(g[f"G_{t}"].reshape(N, Cout, OH, OW))
    dt = torch.float32 if operands == "f32" else torch.bfloat16
    tol = F32_TOL if operands == "f32" else BF16_TOL
    Y = dgx.conv2d(X, K, b, KH, KW, operands=dt)
    dX, dK = dgx.conv2d_backward(X, K, G, KH, KW, operands=dt)
    dgx.sync_check()
    assert normwise(Y.cpu().numpy(), g[f"Y_{t}"].reshape(N, Cout, OH, OW)) < tol
    assert normwise(dX.cpu().numpy(), g[f"dX_{t}"].reshape(N, Cin, H, W)) < tol
    assert normwise(dK.cpu().numpy(), g[f"dK_{t}"]) < tol


@pytest.mark.parametrize("cfg", CONV_PAD_CFGS)
def test_reference_conv2d_padded_and_gradient(dgx, orc, golden, cfg):
    g = golden("conv")
    N, Cin, H, W, Cout, KH, KW, pad, stride = cfg
    t = "p" + "_".join(map(str, cfg))
    OH, OW = orc.conv_out(H, W, KH, KW, pad, stride)
    Xh = g[f"X_{t}"].reshape(N, Cin, H, W)
    X, K, b = cuda(Xh), cuda(g[f"K_{t}"]), cuda(g[f"b_{t}"])
    Y = dgx.conv2d(X, K, b, KH, KW, pad=pad, stride=stride)
    G = np.random.default_rng(sum(cfg)).standard_normal((N, Cout, OH, OW))
    dX, dK = dgx.conv2d_backward(X, K, cuda(G), KH, KW, pad=pad, stride=stride)
    dgx.sync_check()
    assert normwise(Y.cpu().numpy(), g[f"Y_{t}"].reshape(N, Cout, OH, OW)) < F32_TOL
    rdX, rdK = orc.conv2d_bwd(Xh, g[f"K_{t}"], G.astype(np.float32), KH, KW, pad, stride)
    assert normwise(dX.cpu().numpy(), rdX) < F32_TOL
    assert normwise(dK.cpu().numpy(), rdK) < F32_TOL


@pytest.mark.parametrize("operands", ["f32", "bf16"])
def test_conv_layer_sized(dgx, orc, operands):
    """A 3x3, pad 1 layer at network size: 8 x 64 x 32 x 32 -> 128 channels
    (one GEMM of 8192 x 128 x 576), plus a strided 1x1 projection."""
    rng = np.random.default_rng(11)
    for (N, Cin, H, W, Cout, KH, KW, pad, stride) in [(8, 64, 32, 32, 128, 3, 3, 1, 1), (4, 64, 16, 16, 32, 1, 1, 0, 2)]:
        Xh = rng.standard_normal((N, Cin, H, W)).astype(np.float32)
        Kh = (rng.standard_normal((Cout, Cin * KH * KW)) / np.sqrt(Cin * KH * KW)).astype(np.float32)
        bh = rng.standard_normal(Cout).astype(np.float32)
        dt = torch.float32 if operands == "f32" else torch.bfloat16
        tol = F32_TOL if operands == "f32" else BF16_TOL
        Y = dgx.conv2d(cuda(Xh), cuda(Kh), cuda(bh), KH, KW, pad=pad, stride=stride, operands=dt)
        OH, OW = orc.conv_out(H, W, KH, KW, pad, stride)
        G = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
        dX, dK = dgx.conv2d_backward(cuda(Xh), cuda(Kh), cuda(G), KH, KW, pad=pad, stride=stride, operands=dt)
        dgx.sync_check()
        assert normwise(Y.cpu().numpy(), orc.conv2d_fwd(Xh, Kh, bh, KH, KW, pad, stride)) < tol
        rdX, rdK = orc.conv2d_bwd(Xh, Kh, G, KH, KW, pad, stride)
        assert normwise(dX.cpu().numpy(), rdX) < tol
        assert normwise(dK.cpu().numpy(), rdK) < tol


def test_conv_rejects_bad_geometry(dgx):
    X = torch.zeros(1, 1, 3, 3, device="cuda")
    K = torch.zeros(1, 16, device="cuda")
    with pytest.raises(dgx.DgxError):
        dgx.conv2d(X, K, None, 4, 4)  # kernel larger than the input
