"""CPU: the int8 network format of export_c_header_int8
(runtime/nn/training.inc:3494-3817). The fixture is a 3-layer MLP exported by
the reference itself (tests/golden/int8_export/mlp_int8.c) with the outputs
of that emitted C code; the oracle's quantiser and dense_q reproduce both,
and the per-channel exporter of dreamcompiler_b200.int8_export writes a file
that reads back to the same layers."""
import os

import numpy as np
import pytest

from conftest import normwise

from dreamcompiler_b200 import int8_export as IE

HERE = os.path.dirname(os.path.abspath(__file__))
EXPORTED = os.path.join(HERE, "golden", "int8_export", "mlp_int8.c")
NAMES = ["fc1", "fc2", "fc3"]


def oracle_chain(orc, layers, X):
    cur = np.asarray(X, np.float32)
    for L in layers:
        sc = np.full(L.out_dim, L.scale, np.float32) if isinstance(L.scale, float) else L.scale
        cur = orc.dense_q(cur, L.W, sc, L.bias)
        if L.relu:
            cur = np.maximum(cur, 0.0).astype(np.float32)
    return cur


def test_parse_reference_export(orc, golden):
    g = golden("int8_export")
    layers = IE.load_c_file(EXPORTED)
    assert [L.relu for L in layers] == [True, True, False]
    for L, name in zip(layers, NAMES):
        q, s = orc.quantize_per_tensor(g[f"{name}_W"])
        assert np.array_equal(L.W, q), name            # the emitted int8 array, bit for bit
        assert np.float32(L.scale) == np.float32(s)    # emitted as (float)scale, %.9g
        assert np.array_equal(L.bias, g[f"{name}_b"].astype(np.float32))


def test_oracle_chain_matches_emitted_code(orc, golden):
    g = golden("int8_export")
    Y = oracle_chain(orc, IE.load_c_file(EXPORTED), g["X"])
    assert normwise(Y, g["Y"]) < 1e-6


def test_per_channel_exporter(orc, golden, tmp_path):
    g = golden("int8_export")
    layers = [(n, g[f"{n}_W"], g[f"{n}_b"]) for n in NAMES]
    for _, W, _ in layers:
        q, sc = IE.quantize_rows_per_channel(W)
        for j in range(W.shape[0]):  # each row under the exporter's per-tensor rule
            qo, so = orc.quantize_per_tensor(W[j:j + 1])
            assert np.array_equal(q[j], qo[0]) and sc[j] == so
    prefix = str(tmp_path / "mlp_pc")
    IE.export_c_header_int8_per_channel(layers, prefix, "mlp_predict_pc")
    back = IE.load_c_file(prefix + ".c")
    assert [L.relu for L in back] == [True, True, False]
    for L, (_, W, b) in zip(back, layers):
        q, sc = IE.quantize_rows_per_channel(W)
        assert np.array_equal(L.W, q)
        assert np.array_equal(L.scale, sc.astype(np.float32))
        assert np.array_equal(L.bias, b.astype(np.float32))
    assert normwise(oracle_chain(orc, back, g["X"]), g["Ypc"]) < 1e-6
    # per-channel scales track each row's range: no worse than the per-tensor export
    assert normwise(g["Ypc"], g["Y"]) < 0.05


def test_parser_rejects_other_files():
    with pytest.raises(ValueError):
        IE.parse_c_source("int main(void) { return 0; }")
    bad = open(EXPORTED).read().replace("static const int8_t fc1_weight[1920]", "static const int8_t fc1_weight[1921]")
    with pytest.raises(ValueError):
        IE.parse_c_source(bad)
