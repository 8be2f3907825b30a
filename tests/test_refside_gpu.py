"""GPU: the reference Dream runtime itself, built with the B200 backend
(dreamcompiler_b200/refside: b200.inc included after runtime/backend/gpu.inc,
libdgx linked). The programs below are the golden-vector generator's own
programs, run through the reference's ops on the reference's struct Tensor;
results are compared with what the unmodified reference computed on the CPU
(tests/golden/). Float64 tensors now compute in f64 on the device, so the
GEMM gates are 1e-12; FlashAttention runs on bf16 operands (1e-2 class)."""
import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def R():
    from dreamcompiler_b200 import refside
    if not refside.available():
        pytest.fail("libdream_ref_b200.so is not built (dreamcompiler_b200/refside/build.sh)")
    refside.load()
    return refside


def seeded_backward(R, out, shape):
    g = R.call("dream_randn", R.scalar(shape[0]), R.scalar(shape[1]))
    R.call("backward", R.call("sum", R.call("tensor_mul", out, g)))
    return R.data(g)


def test_matmul_program(R, golden):
    """set_seed(42); per gemm_selftest shape: A, B = randn; C = A @ B;
    backward(sum(C * randn)) on the device in f64."""
    g = golden("gemm")
    before = R.counts()
    R.call("dream_set_seed", R.scalar(42))
    shapes = [(1, 1, 1), (1, 7, 1), (5, 1, 9), (3, 4, 5), (7, 13, 17), (31, 33, 37), (64, 64, 64), (65, 63, 66),
              (128, 100, 96)]
    for (M, K, N) in shapes:
        t = f"{M}x{K}x{N}"
        A = R.call("dream_randn", R.scalar(M), R.scalar(K))
        B = R.call("dream_randn", R.scalar(K), R.scalar(N))
        assert np.array_equal(R.data(A), g[f"A_{t}"])
        C = R.call("tensor_matmul", A, B)
        G = seeded_backward(R, C, (M, N))
        assert np.array_equal(G, g[f"G_{t}"])
        assert normwise(R.data(C), g[f"C_{t}"]) < 1e-12, t
        assert normwise(R.grad(A), g[f"dA_{t}"]) < 1e-12, t
        assert normwise(R.grad(B), g[f"dB_{t}"]) < 1e-12, t
    after = R.counts()
    assert after["matmul_f64"] - before["matmul_f64"] == len(shapes)
    assert after["matmul_bwd"] - before["matmul_bwd"] == len(shapes)


def test_linear_program(R, golden):
    g = golden("linear")
    before = R.counts()
    R.call("dream_set_seed", R.scalar(11))
    for relu in (0, 1):
        for (N, din, dout) in [(8, 16, 12), (33, 65, 17)]:
            t = f"{relu}_{N}_{din}_{dout}"
            X, W, b = (R.call("dream_randn", R.scalar(r), R.scalar(c)) for r, c in ((N, din), (dout, din), (1, dout)))
            Y = R.call("dream_linear_relu" if relu else "dream_linear", X, W, b)
            seeded_backward(R, Y, (N, dout))
            assert normwise(R.data(Y), g[f"Y_{t}"]) < 1e-12
            assert normwise(R.grad(X), g[f"dX_{t}"]) < 1e-12
            assert normwise(R.grad(W), g[f"dW_{t}"]) < 1e-12
            assert normwise(R.grad(b)[0], g[f"db_{t}"]) < 1e-12
    after = R.counts()
    assert after["linear"] - before["linear"] == 4 and after["linear_bwd"] - before["linear_bwd"] == 4


def test_flash_program(R, golden):
    g = golden("flash")
    before = R.counts()
    R.call("dream_set_seed", R.scalar(20260709))
    cfgs = [(64, 16, 8), (64, 16, 16), (128, 32, 32), (100, 24, 16), (128, 64, 64), (160, 64, 32)]
    for (S, dk, Bc) in cfgs:
        B = 2 if S * dk <= 4096 else 1
        t = f"{S}_{dk}_{Bc}"
        Q, K, V = (R.call("dream_randn", R.scalar(B), R.scalar(S * dk)) for _ in range(3))
        O = R.call("dream_flash_attention", Q, K, V, R.scalar(B), R.scalar(S), R.scalar(dk), R.scalar(Bc))
        seeded_backward(R, O, (B, S * dk))
        shape = (B, S, dk)
        assert normwise(R.data(O, shape), g[f"O_{t}"]) < 2e-2, t
        for name, x in (("dQ", Q), ("dK", K), ("dV", V)):
            assert normwise(R.grad(x, shape), g[f"{name}_{t}"]) < 2e-2, (t, name)
    after = R.counts()
    assert after["flash_fwd"] - before["flash_fwd"] == len(cfgs)
    assert after["flash_bwd"] - before["flash_bwd"] == len(cfgs)


def test_tensor_parallel_selftest(R):
    """The reference's own tensor_parallel_selftest (training.inc:1668-1700):
    column- and row-split matmuls through tensor_matmul on the device equal the
    un-split one (1e-12 / 1e-10, its own gates)."""
    before = R.counts()["matmul_f64"]
    assert R.data(R.call("tensor_parallel_selftest"))[0, 0] == 1.0
    assert R.counts()["matmul_f64"] > before


def test_tp_matmul_column_goldens(R, golden):
    g = golden("tp")
    for (M, K, N) in [(12, 16, 24), (9, 10, 23)]:
        X, W = R.tensor(g[f"X_{M}_{K}_{N}"]), R.tensor(g[f"W_{M}_{K}_{N}"])
        for G in (1, 2, 3, 4, 5, 7):
            Y = R.call("dream_tp_matmul_column", X, W, R.scalar(G))
            assert normwise(R.data(Y), g[f"Y_{M}_{K}_{N}_{G}"]) < 1e-12


def test_f32_precision_path(R):
    """`as f32` operands take the float32 branch (3xTF32 on the device), with
    the reference's bookkeeping: tests/10_f32_matmul.dream, sum(ones@ones) == 8."""
    a = R.tensor(np.ones((2, 2)))
    R.call("dream_set_precision", a, 1)
    before = R.counts()["matmul_f32"]
    c = R.call("tensor_matmul", a, a)
    assert R.data(R.call("sum", c))[0, 0] == 8.0
    assert R.counts()["matmul_f32"] == before + 1
    rng = np.random.default_rng(1)
    A, B = rng.standard_normal((100, 70)), rng.standard_normal((70, 90))
    ta, tb = R.tensor(A), R.tensor(B)
    R.call("dream_set_precision", ta, 1)
    R.call("dream_set_precision", tb, 1)
    tc = R.call("tensor_matmul", ta, tb)
    ref = A.astype(np.float32).astype(np.float64) @ B.astype(np.float32).astype(np.float64)
    assert normwise(R.data(tc), ref) < 1e-5


def test_chained_ops_reuse_device_copies(R):
    """C = A @ B; D = C @ E: C's device copy from the first op feeds the
    second (no upload). A host-side change to C fails its fingerprint and is
    uploaded again, so the result follows the host data."""
    rng = np.random.default_rng(2)
    A, B, E = rng.standard_normal((64, 48)), rng.standard_normal((48, 80)), rng.standard_normal((80, 32))
    ta, tb, te = R.tensor(A), R.tensor(B), R.tensor(E)
    tc = R.call("tensor_matmul", ta, tb)
    c0 = R.counts()
    td = R.call("tensor_matmul", tc, te)
    c1 = R.counts()
    assert c1["uploads"] - c0["uploads"] == 1          # E only
    assert c1["mirror_hits"] - c0["mirror_hits"] == 1  # C
    assert normwise(R.data(td), (A @ B) @ E) < 1e-12
    R.view(tc)[5] += 1.0                                # in-place host change
    td2 = R.call("tensor_matmul", tc, te)
    c2 = R.counts()
    assert c2["uploads"] - c1["uploads"] == 1          # C again; E reused
    Cm = A @ B
    Cm.flat[5] += 1.0
    assert normwise(R.data(td2), Cm @ E) < 1e-12


def test_error_behaviour_is_the_references(R, capfd):
    a = R.call("alloc_tensor", 2, 3, 1, 1)
    b = R.call("alloc_tensor", 4, 2, 1, 1)
    c = R.call("tensor_matmul", a, b)
    assert (c.contents.d0, c.contents.d1) == (1, 1)
    assert "RUNTIME ERROR in matmul (@)" in capfd.readouterr().err
