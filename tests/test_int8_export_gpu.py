"""GPU: exported int8 networks run batched on the device (dgx_dense_q per
layer) against the outputs of the reference's emitted C code and the
oracle. Tolerance: normwise 1e-5 (the device products are exact and rounded
once per output; the emitted code adds fp32 terms one by one)."""
import os

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from dreamcompiler_b200 import int8_export as IE  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
EXPORTED = os.path.join(HERE, "golden", "int8_export", "mlp_int8.c")
TOL = 1e-5


def run(net, X):
    return net.predict(torch.from_numpy(np.ascontiguousarray(X, np.float32)).cuda()).cpu().numpy()


def test_reference_export_on_device(dgx, golden):
    g = golden("int8_export")
    net = IE.Int8Net.from_c_file(EXPORTED)
    Y = run(net, g["X"])
    dgx.sync_check()
    assert normwise(Y, g["Y"]) < TOL


def test_per_channel_export_on_device(dgx, golden, tmp_path):
    g = golden("int8_export")
    layers = [(n, g[f"{n}_W"], g[f"{n}_b"]) for n in ("fc1", "fc2", "fc3")]
    prefix = str(tmp_path / "mlp_pc")
    IE.export_c_header_int8_per_channel(layers, prefix, "mlp_predict_pc")
    Y = run(IE.Int8Net.from_c_file(prefix + ".c"), g["X"])
    dgx.sync_check()
    assert normwise(Y, g["Ypc"]) < TOL


@pytest.mark.parametrize("per_channel", [False, True])
def test_wide_network_tensor_core_path(dgx, orc, tmp_path, per_channel):
    """4096 -> 1024 -> 16 (K multiple of 16: the tensor-core kernel), batch
    of 64, written by the exporters' quantisers and read back."""
    rng = np.random.default_rng(7)
    layers = [("l1", rng.standard_normal((1024, 4096)) * 0.02, rng.standard_normal(1024) * 0.1),
              ("l2", rng.standard_normal((16, 1024)) * 0.05, rng.standard_normal(16) * 0.1)]
    if per_channel:
        prefix = str(tmp_path / "wide")
        IE.export_c_header_int8_per_channel(layers, prefix, "wide_predict")
        net_layers = IE.load_c_file(prefix + ".c")
    else:
        net_layers = []
        for i, (name, W, b) in enumerate(layers):
            q, s = orc.quantize_per_tensor(W)
            net_layers.append(IE.Int8Layer(name, q, float(np.float32(s)), b.astype(np.float32), i == 0))
    X = rng.standard_normal((64, 4096)).astype(np.float32)
    Y = run(IE.Int8Net(net_layers), X)
    dgx.sync_check()
    cur = X
    for L in net_layers:
        sc = np.full(L.out_dim, L.scale, np.float32) if isinstance(L.scale, float) else L.scale
        cur = orc.dense_q(cur, L.W, sc, L.bias)
        cur = np.maximum(cur, 0).astype(np.float32) if L.relu else cur
    assert normwise(Y, cur) < TOL


def test_dense_q_relu_flag_and_errors(dgx):
    from dreamcompiler_b200 import _lib as L
    X = torch.randn(4, 64, device="cuda")
    W = torch.randint(-127, 128, (32, 64), device="cuda", dtype=torch.int8)
    b = torch.randn(32, device="cuda")
    y0 = torch.empty(4, 32, device="cuda")
    y1 = torch.empty(4, 32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L.call("dgx_dense_q", X.data_ptr(), W.data_ptr(), 0.01, None, b.data_ptr(), y0.data_ptr(), 4, 32, 64, 0, s)
    L.call("dgx_dense_q", X.data_ptr(), W.data_ptr(), 0.01, None, b.data_ptr(), y1.data_ptr(), 4, 32, 64, 1, s)
    dgx.sync_check()
    assert (y0 < 0).any() and torch.equal(y1, torch.clamp(y0, min=0))
    with pytest.raises(dgx.DgxError):
        L.call("dgx_dense_q", X.data_ptr(), None, 0.01, None, b.data_ptr(), y0.data_ptr(), 4, 32, 64, 0, s)
