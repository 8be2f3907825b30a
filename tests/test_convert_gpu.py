"""GPU: dgx_convert's bf16 rounding, bit for bit against the reference's
dream_to_bf16 (runtime/nn/training.inc:1969-1976) as the oracle restates it
(orc.bf16_bits). Every Dream op on the bf16 path uploads its operands through
this converter, so its bits are the operands' bits.

Cases: every sign/exponent/high-mantissa pattern with the dropped half at the
rounding boundaries (ties to even, one below and above a tie, carries into
the exponent and into infinity), +-0, subnormals, +-inf, NaNs (including the
payloads the reference's integer rounding turns into infinity or wraps to
zero), random bit patterns, and f64 inputs whose f64 -> f32 step decides the
bf16 tie."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _convert(src: "torch.Tensor", src_type: int, n: int):
    from dreamcompiler_b200 import _lib
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("dgx_convert", src.data_ptr(), src_type, out.data_ptr(), _lib.DGX_BF16, n, 0, s)
    _lib.check(_lib.load().dgx_sync_check(s), "dgx_sync_check")
    return out.cpu().numpy().view(np.uint16)


def _f32_patterns():
    hi = np.arange(1 << 16, dtype=np.uint32) << 16
    lows = np.array([0x0000, 0x0001, 0x7FFF, 0x8000, 0x8001, 0xFFFF], np.uint32)
    edge = (hi[:, None] | lows[None, :]).ravel()
    named = np.array([0x00000000, 0x80000000, 0x00000001, 0x00008000, 0x00018000, 0x007FFFFF, 0x807FFFFF,
                      0x3F7FFFFF, 0x3F808000, 0x3F818000, 0x7F7FFFFF, 0x7F7F8000, 0xFF7FFFFF,
                      0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001, 0x7F808000,
                      0xFFFF8000, 0xFFFFFFFF, 0x7FFFFFFF], np.uint32)
    rnd = np.random.default_rng(1).integers(0, 1 << 32, 1 << 22, dtype=np.uint64).astype(np.uint32)
    return np.concatenate([named, edge, rnd])


def test_f32_to_bf16_bits_match_the_reference(dgx, orc):
    bits = _f32_patterns()
    x = bits.view(np.float32)
    got = _convert(torch.from_numpy(x.copy()).cuda(), 0, x.size)
    ref = orc.bf16_bits(x)
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, [(hex(bits[i]), hex(got[i]), hex(ref[i])) for i in bad[:8]]


def test_f64_to_bf16_rounds_through_f32_like_the_reference(dgx, orc):
    rng = np.random.default_rng(2)
    # f32 values exactly on a bf16 tie, then nudged by less than half an f32
    # ulp: f64 -> f32 lands on the tie, which then rounds to even (a direct
    # f64 -> bf16 rounding would go the other way for the upward nudges).
    tie_bits = ((rng.integers(0x0080, 0x7F7F, 1 << 16, dtype=np.uint32) << 16) | 0x8000).astype(np.uint32)
    ties = tie_bits.view(np.float32).astype(np.float64)
    ulp = np.abs(ties) * 2.0 ** -24
    nudged = np.concatenate([ties, ties + 0.25 * ulp, ties - 0.25 * ulp, -(ties + 0.25 * ulp),
                             ties + 0.75 * ulp])
    wide = rng.standard_normal(1 << 20) * np.exp2(rng.integers(-140, 120, 1 << 20))
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-310, -1e-310, 3.5e38, -3.5e38, 1e300, 2.0 ** -149,
                        2.0 ** -150, 2.0 ** -151])
    x = np.concatenate([nudged, wide, special])
    got = _convert(torch.from_numpy(x).cuda(), 3, x.size)
    with np.errstate(over="ignore"):
        ref = orc.bf16_bits(x.astype(np.float32))  # numpy's f64 -> f32 cast rounds to nearest even
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, [(repr(x[i]), hex(got[i]), hex(ref[i])) for i in bad[:8]]


def test_widening_conversions_are_exact(dgx):
    from dreamcompiler_b200 import _lib
    rng = np.random.default_rng(3)
    n = 1 << 16
    b16 = torch.from_numpy(rng.integers(0, 1 << 16, n, dtype=np.uint16).view(np.int16)).cuda()
    f32 = torch.empty(n, dtype=torch.float32, device="cuda")
    f64 = torch.empty(n, dtype=torch.float64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("dgx_convert", b16.data_ptr(), _lib.DGX_BF16, f32.data_ptr(), _lib.DGX_F32, n, 0, s)
    _lib.call("dgx_convert", f32.data_ptr(), _lib.DGX_F32, f64.data_ptr(), _lib.DGX_F64, n, 0, s)
    _lib.check(_lib.load().dgx_sync_check(s), "dgx_sync_check")
    want = (b16.cpu().numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    got32 = f32.cpu().numpy()
    assert np.array_equal(got32.view(np.uint32)[~np.isnan(want)], want.view(np.uint32)[~np.isnan(want)])
    assert np.isnan(got32[np.isnan(want)]).all()
    got64 = f64.cpu().numpy()
    assert np.array_equal(got64[~np.isnan(want)], want.astype(np.float64)[~np.isnan(want)])
