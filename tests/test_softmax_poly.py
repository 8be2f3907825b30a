"""CPU: the polynomial 2^x that the FlashAttention forward uses for part of
its exponentials (flash_fwd.cu, ex2_poly2), evaluated here in float32 (the
device fuses each multiply-add): its relative error over the softmax's
argument range stays far below the 3.9e-3 resolution of the bf16 P it feeds."""
import numpy as np


def ex2_poly(x):
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x - j).astype(np.float32)
    p = (np.float32(0.05517166) * f + np.float32(0.24261113)).astype(np.float32)
    p = (p * f + np.float32(0.69326097)).astype(np.float32)
    p = (p * f + np.float32(0.99992806)).astype(np.float32)
    return (p.view(np.int32) + (t.view(np.int32) << 23)).view(np.float32)


def test_relative_error_over_the_softmax_range():
    x = np.linspace(-60.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 1e-4


def test_masked_scores_are_negligible():
    assert ex2_poly(np.array([-np.inf], np.float32))[0] < 2e-38
