"""CPU: the GPT-step oracle (oracle/gpt_oracle.py) against golden vectors the
reference runtime produced (tests/golden/make_golden.py: one training step of
the config-3 architecture composed from the reference's own ops, and
dream_adamw_update)."""
import os

import numpy as np

from oracle import gpt_oracle as G

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_step_matches_reference_runtime():
    z = np.load(os.path.join(GOLD, "gpt.npz"))
    L, d, H, B, S, V, _ = (int(x) for x in z["cfg"])
    params = {k[2:]: z[k] for k in z.files if k.startswith("p_")}
    loss, grads = G.step(params, z["tok"], z["tgt"], L, d, H, B, S, V)
    assert abs(loss - float(z["loss"])) <= 1e-12 * abs(float(z["loss"]))
    assert set(grads) == set(params)
    for k, g in grads.items():
        ref = z["g_" + k].astype(np.float64)
        # the fixture stores gradients as float32
        assert np.linalg.norm(g - ref) <= 1e-6 * np.linalg.norm(ref), k


def test_adamw_matches_reference_runtime():
    a = np.load(os.path.join(GOLD, "adamw.npz"))
    p, m, v = a["p0"], np.zeros_like(a["p0"]), np.zeros_like(a["p0"])
    for k in (1, 2):
        p, m, v = G.adamw(p, a[f"g{k}"], m, v, k, 3e-4)
        np.testing.assert_allclose(p, a[f"p{k}"], rtol=0, atol=1e-15)


def test_init_is_seeded():
    a = G.init_params(2, 32, 65, 16, 5)
    b = G.init_params(2, 32, 65, 16, 5)
    assert all(np.array_equal(a[k], b[k]) for k in a)
    assert set(a) == set(G.param_shapes(2, 32, 65, 16))
