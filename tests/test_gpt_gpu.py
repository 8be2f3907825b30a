"""GPU: the device-resident GPT training step (BASELINE config 3
architecture) against the reference runtime's own step (golden vectors from
tests/golden/make_golden.py) and the f64 oracle (oracle/gpt_oracle.py).

The device step runs its GEMMs and attention on bf16 operands with fp32
accumulation (fp32 master weights, activations and gradients elsewhere), the
reference in f64: the loss must agree to 1e-3 relative and every parameter's
gradient to 1e-2 normwise (the bf16 tolerance of the task; measured: 7e-6 and <5e-3)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle import gpt_oracle as G  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")
LOSS_RTOL, GRAD_TOL = 1e-3, 1e-2


def _grads(model, names):
    V = model.cfg.vocab
    out = {}
    for k in names:
        gk = model.g[k].float().cpu().numpy()
        out[k] = gk[:V] if k in ("Wout", "bout") else gk
    return out


def _check(model, loss_ref, grads_ref, report=None):
    loss = float(model.loss.item())
    errs = {}
    got = _grads(model, grads_ref)
    for k, ref in grads_ref.items():
        ref = np.asarray(ref, np.float64).reshape(got[k].shape)
        errs[k] = np.linalg.norm(got[k] - ref) / np.linalg.norm(ref)
    if report is not None:
        report.update(errs)
    assert abs(loss - loss_ref) <= LOSS_RTOL * abs(loss_ref), (loss, loss_ref)
    bad = {k: e for k, e in errs.items() if not e <= GRAD_TOL}
    assert not bad, bad


def test_step_matches_reference_runtime_golden(dgx):
    from dreamcompiler_b200.gpt import GPT, GPTConfig
    z = np.load(os.path.join(GOLD, "gpt.npz"))
    L, d, H, B, S, V, _ = (int(x) for x in z["cfg"])
    params = {k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("p_")}
    m = GPT(GPTConfig(n_layer=L, d_model=d, n_head=H, seq_len=S, batch=B, vocab=V), params=params)
    m.set_batch(torch.from_numpy(z["tok"]), torch.from_numpy(z["tgt"]))
    m.forward_backward()
    dgx.sync_check()
    _check(m, float(z["loss"]), {k[2:]: z[k] for k in z.files if k.startswith("g_")})


@pytest.mark.parametrize("L,d,H,B,S", [(2, 128, 2, 2, 128), (1, 192, 3, 3, 256)])
def test_step_matches_oracle(dgx, L, d, H, B, S):
    from dreamcompiler_b200.gpt import GPT, GPTConfig
    V = 65
    params = G.init_params(L, d, V, S, seed=L * 100 + d)
    rng = np.random.default_rng(d)
    tok, tgt = rng.integers(0, V, B * S), rng.integers(0, V, B * S)
    loss_ref, grads_ref = G.step(params, tok, tgt, L, d, H, B, S, V)
    m = GPT(GPTConfig(n_layer=L, d_model=d, n_head=H, seq_len=S, batch=B, vocab=V),
            params={k: torch.from_numpy(v) for k, v in params.items()})
    m.set_batch(torch.from_numpy(tok.astype(np.int32)), torch.from_numpy(tgt.astype(np.int32)))
    m.forward_backward()
    dgx.sync_check()
    _check(m, loss_ref, grads_ref)


def test_adamw_kernel_matches_oracle(dgx):
    from dreamcompiler_b200 import _lib
    rng = np.random.default_rng(4)
    p0, g1, g2 = (rng.standard_normal(10000) for _ in range(3))
    p = torch.from_numpy(p0.astype(np.float32)).cuda()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    step_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    pr, mr, vr = p0.astype(np.float32).astype(np.float64), np.zeros(10000), np.zeros(10000)
    s = torch.cuda.current_stream().cuda_stream
    for k, g in enumerate((g1, g2), 1):
        gd = torch.from_numpy(g.astype(np.float32)).cuda()
        if k == 1:  # host step count
            _lib.call("dgx_adamw", p.data_ptr(), gd.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), 3e-4, 0.9, 0.999,
                      1e-8, 0.01, 1, None, s)
        else:  # device step count
            step_dev.fill_(2)
            _lib.call("dgx_adamw", p.data_ptr(), gd.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), 3e-4, 0.9, 0.999,
                      1e-8, 0.01, 0, step_dev.data_ptr(), s)
        pr, mr, vr = G.adamw(pr, g.astype(np.float32).astype(np.float64), mr, vr, k, 3e-4)
        assert not gd.any().item()  # gradient zeroed
    dgx.sync_check()
    np.testing.assert_allclose(p.cpu().numpy(), pr, rtol=0, atol=2e-6)


def test_training_reduces_loss(dgx):
    from dreamcompiler_b200.gpt import GPT, GPTConfig
    cfg = GPTConfig(n_layer=2, d_model=128, n_head=2, seq_len=128, batch=4, vocab=65, lr=1e-3)
    m = GPT(cfg, seed=1)
    g = torch.Generator().manual_seed(2)
    tok = torch.randint(0, 65, (cfg.batch * cfg.seq_len,), generator=g, dtype=torch.int32)
    m.set_batch(tok, torch.roll(tok, -1))  # learnable: next token of a fixed sequence
    first = None
    for i in range(30):
        loss = m.step()
        if i == 0:
            first = loss.item()
    dgx.sync_check()
    assert loss.item() < 0.8 * first, (first, loss.item())


@pytest.mark.parametrize("n", [8 * 1000, 8 * 1000 + 5, 3])
def test_gelu_kernels_against_oracle(dgx, n):
    """dgx_gelu_fwd / dgx_gelu_bwd on bf16 (the 8-wide vector kernel plus the
    scalar tail) against the oracle's f64 GELU (runtime/io/builtins.inc:548-560)
    and its derivative (runtime/ops/autograd.inc:293-303) of the same bf16
    inputs; tolerance 1e-2 normwise (bf16 output)."""
    from dreamcompiler_b200 import _lib as L
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(n, device="cuda", generator=g) * 3).bfloat16()
    dy = torch.randn(n, device="cuda", generator=g).bfloat16()
    y = torch.empty_like(x)
    dx = torch.empty_like(x)
    s = torch.cuda.current_stream().cuda_stream
    L.call("dgx_gelu_fwd", x.data_ptr(), L.DGX_BF16, y.data_ptr(), n, s)
    L.call("dgx_gelu_bwd", x.data_ptr(), L.DGX_BF16, dy.data_ptr(), L.DGX_BF16, dx.data_ptr(), n, s)
    dgx.sync_check()
    xf, df = x.double().cpu().numpy(), dy.double().cpu().numpy()
    ry, rdx = G.gelu(xf), G.gelu_bwd(xf, df)
    nw = lambda a, r: np.abs(a - r).max() / max(np.abs(r).max(), 1e-30)
    assert nw(y.double().cpu().numpy(), ry) < 1e-2
    assert nw(dx.double().cpu().numpy(), rdx) < 1e-2


@pytest.mark.parametrize("C", [384, 1024, 100])
def test_layernorm_kernels_against_oracle(dgx, C):
    """dgx_layernorm_fwd / dgx_layernorm_bwd (row-in-registers path for C a
    multiple of 128, scalar path otherwise) against the f64 oracle's
    layer_norm and its backward (runtime/io/builtins.inc:167-197,
    runtime/ops/autograd.inc:453-470): y16 to the bf16 tolerance, mean,
    rstd and dx to 1e-5 normwise."""
    from dreamcompiler_b200 import _lib as L
    R = 777
    g = torch.Generator(device="cuda").manual_seed(C)
    x = torch.randn(R, C, device="cuda", generator=g) * 2 + 0.5
    dy = torch.randn(R, C, device="cuda", generator=g)
    y16 = torch.empty(R, C, device="cuda", dtype=torch.bfloat16)
    mu, rs = torch.empty(R, device="cuda"), torch.empty(R, device="cuda")
    dx = torch.empty(R, C, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L.call("dgx_layernorm_fwd", x.data_ptr(), y16.data_ptr(), mu.data_ptr(), rs.data_ptr(), R, C, s)
    L.call("dgx_layernorm_bwd", x.data_ptr(), mu.data_ptr(), rs.data_ptr(), dy.data_ptr(), dx.data_ptr(), R, C, 0, s)
    dgx.sync_check()
    xf, dyf = x.double().cpu().numpy(), dy.double().cpu().numpy()
    ry, inv = G.layer_norm(xf)
    rdx = G.layer_norm_bwd(ry, inv, dyf)
    nw = lambda a, r: np.abs(a - r).max() / np.abs(r).max()
    assert nw(y16.double().cpu().numpy(), ry) < 1e-2
    assert nw(rs.double().cpu().numpy(), np.asarray(inv).reshape(-1)) < 1e-5
    assert nw(mu.double().cpu().numpy(), xf.mean(1)) < 1e-5
    assert nw(dx.double().cpu().numpy(), rdx) < 1e-5


@pytest.mark.parametrize("accumulate", [0, 1])
def test_layernorm_bwd_x16_matches_separate_conversion(dgx, accumulate):
    """dgx_layernorm_bwd_x16: the same fp32 dx as dgx_layernorm_bwd, plus
    dx16 = bf16(dx) bit for bit (what converting dx afterwards gives)."""
    from dreamcompiler_b200 import _lib as L
    R, C = 1000, 384
    g = torch.Generator(device="cuda").manual_seed(17 + accumulate)
    x, dy, dx0 = (torch.randn(R, C, device="cuda", generator=g) for _ in range(3))
    y16 = torch.empty(R, C, device="cuda", dtype=torch.bfloat16)
    mu, rs = torch.empty(R, device="cuda"), torch.empty(R, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L.call("dgx_layernorm_fwd", x.data_ptr(), y16.data_ptr(), mu.data_ptr(), rs.data_ptr(), R, C, s)
    dx_a, dx_b = dx0.clone(), dx0.clone()
    dx16 = torch.empty(R, C, device="cuda", dtype=torch.bfloat16)
    L.call("dgx_layernorm_bwd", x.data_ptr(), mu.data_ptr(), rs.data_ptr(), dy.data_ptr(), dx_a.data_ptr(), R, C,
           accumulate, s)
    L.call("dgx_layernorm_bwd_x16", x.data_ptr(), mu.data_ptr(), rs.data_ptr(), dy.data_ptr(), dx_b.data_ptr(),
           dx16.data_ptr(), R, C, accumulate, s)
    dgx.sync_check()
    assert torch.equal(dx_a, dx_b)
    assert torch.equal(dx16, dx_a.bfloat16())


@pytest.mark.parametrize("dtype,R,N", [("bf16", 16384, 1536), ("bf16", 16384, 384), ("f32", 16384, 65),
                                       ("f32", 1000, 384), ("bf16", 77, 24)])
def test_colsum_kernels(dgx, dtype, R, N):
    """dgx_colsum (bias gradients: column sums of dY, fixed-order slices) on
    the vector path (16-byte rows) and the scalar one, with accumulate."""
    from dreamcompiler_b200 import _lib as L
    g = torch.Generator(device="cuda").manual_seed(R + N)
    dy = torch.randn(R, N, device="cuda", generator=g)
    if dtype == "bf16":
        dy = dy.bfloat16()
    db = torch.ones(N, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    t = L.DGX_BF16 if dtype == "bf16" else L.DGX_F32
    L.call("dgx_colsum", dy.data_ptr(), t, db.data_ptr(), R, N, 1, s)
    dgx.sync_check()
    ref = dy.double().sum(0).cpu().numpy() + 1.0
    got = db.double().cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-5


@pytest.mark.parametrize("src_type", ["bf16", "f32"])
def test_head_layout_kernels(dgx, src_type):
    """dgx_rows_to_heads / dgx_heads_to_rows: [B*S][ld] rows (head h at
    column col0 + h*D) <-> [B*H][S][D] heads, bit-exact moves (bf16 source)
    and round-to-nearest for fp32 rows."""
    from dreamcompiler_b200 import _lib as L
    B, S, H, D, ld, col0 = 3, 40, 4, 64, 3 * 256 + 8, 256
    g = torch.Generator(device="cuda").manual_seed(9)
    rows = torch.randn(B * S, ld, device="cuda", generator=g)
    if src_type == "bf16":
        rows = rows.bfloat16()
    heads = torch.empty(B * H, S, D, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    t = L.DGX_BF16 if src_type == "bf16" else L.DGX_F32
    L.call("dgx_rows_to_heads", rows.data_ptr(), t, ld, col0, heads.data_ptr(), B, S, H, D, s)
    back = torch.zeros(B * S, ld, device="cuda", dtype=torch.bfloat16)
    L.call("dgx_heads_to_rows", heads.data_ptr(), back.data_ptr(), ld, col0, B, S, H, D, s)
    dgx.sync_check()
    ref = rows[:, col0:col0 + H * D].bfloat16().reshape(B, S, H, D).permute(0, 2, 1, 3).reshape(B * H, S, D)
    assert torch.equal(heads, ref)
    assert torch.equal(back[:, col0:col0 + H * D], rows[:, col0:col0 + H * D].bfloat16())
    assert not back[:, :col0].any()
