"""The int8 network format of the reference's exporter, on the B200.

`export_c_header_int8` (heellowdsf/DreamCompiler runtime/nn/training.inc:
3494-3817) writes a self-contained C99 file: per layer a
``static const int8_t <layer>_weight[out*in]`` array ([out][in], row = output
channel), one per-tensor ``static const float <layer>_weight_scale``, a
``static const float <layer>_bias[out]`` array, and a predict function that
chains ``dense_q`` calls with ``relu_inplace`` after every layer but the
last.

This module

* reads such a file (`parse_c_source`) into its layers, exactly as emitted;
* runs the network for a whole batch of inputs on the device, one
  `dgx_dense_q` call per layer (`Int8Net.predict`);
* writes the per-output-channel variant of the format
  (`export_c_header_int8_per_channel`): one scale per weight row, quantised
  with the exporter's own rule per row, and a ``dense_qc`` helper taking
  the scale array. `parse_c_source` reads both forms.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np


@dataclass
class Int8Layer:
    name: str                       # the weight array's C name
    W: np.ndarray                   # int8 [out, in]
    scale: Union[float, np.ndarray]  # per-tensor float, or float32 [out] per channel
    bias: np.ndarray                # float32 [out]
    relu: bool                      # relu_inplace follows this layer

    @property
    def out_dim(self) -> int:
        return self.W.shape[0]

    @property
    def in_dim(self) -> int:
        return self.W.shape[1]


_ARRAY = re.compile(r"static const (int8_t|float) (\w+)\[(\d+)\] = \{([^}]*)\};")
_SCALAR = re.compile(r"static const float (\w+) = ([^;]+);")
_CALL = re.compile(r"(dense_qc?)\(cur_in, cur_dim, (\w+), (\w+), (\w+), (\w+), (\d+)\);")


def _floats(body: str) -> np.ndarray:
    return np.array([float(t.strip().rstrip("f")) for t in body.split(",") if t.strip()], np.float32)


def parse_c_source(text: str) -> List[Int8Layer]:
    """Layers of an exported int8 network, in the predict function's order."""
    arrays = {}
    for kind, name, n, body in _ARRAY.findall(text):
        if kind == "int8_t":
            vals = np.array([int(t) for t in body.split(",") if t.strip()], np.int64)
            if vals.min(initial=0) < -128 or vals.max(initial=0) > 127:
                raise ValueError(f"{name}: values outside int8")
            arrays[name] = vals.astype(np.int8)
        else:
            arrays[name] = _floats(body)
        if arrays[name].size != int(n):
            raise ValueError(f"{name}: {arrays[name].size} values, declared {n}")
    scalars = {name: np.float32(float(v.strip().rstrip("f"))) for name, v in _SCALAR.findall(text)}
    body = text[text.index("(const float* input, float* output)"):] if "(const float* input, float* output)" in text \
        else text
    calls = list(_CALL.finditer(body))
    if not calls:
        raise ValueError("no dense_q calls: not an export_c_header_int8 file")
    layers = []
    for i, m in enumerate(calls):
        fn, w, s, b, dst, out = m.groups()
        out = int(out)
        W = arrays[w]
        if W.size % out:
            raise ValueError(f"{w}: {W.size} weights do not split into {out} rows")
        if fn == "dense_q":
            scale: Union[float, np.ndarray] = float(scalars[s])
        else:
            scale = arrays[s]
            if scale.size != out:
                raise ValueError(f"{s}: {scale.size} scales for {out} channels")
        nxt = body[m.end(): calls[i + 1].start() if i + 1 < len(calls) else len(body)]
        relu = f"relu_inplace({dst}, {out});" in nxt
        layers.append(Int8Layer(w, W.reshape(out, -1), scale, arrays[b], relu))
    for a, b in zip(layers, layers[1:]):
        if a.out_dim != b.in_dim:
            raise ValueError(f"{a.name} -> {b.name}: {a.out_dim} outputs feed {b.in_dim} inputs")
    return layers


def load_c_file(path: str) -> List[Int8Layer]:
    with open(path) as f:
        return parse_c_source(f.read())


class Int8Net:
    """An exported int8 network resident on the device; `predict` runs a
    batch through it, one dgx_dense_q launch per layer."""

    def __init__(self, layers: Sequence[Int8Layer], device="cuda"):
        import torch
        self.torch = torch
        self.layers = list(layers)
        self.device = torch.device(device)
        self.W = [torch.from_numpy(np.ascontiguousarray(L.W)).to(self.device) for L in self.layers]
        self.b = [torch.from_numpy(np.ascontiguousarray(L.bias, np.float32)).to(self.device) for L in self.layers]
        self.s = [None if isinstance(L.scale, float) else
                  torch.from_numpy(np.ascontiguousarray(L.scale, np.float32)).to(self.device) for L in self.layers]

    @classmethod
    def from_c_file(cls, path: str, device="cuda") -> "Int8Net":
        return cls(load_c_file(path), device)

    def predict(self, X):
        """X: [B, in_dim] float32 on the device -> [B, out_dim] float32."""
        from . import _lib as L
        torch = self.torch
        assert X.dtype == torch.float32 and X.dim() == 2 and X.shape[1] == self.layers[0].in_dim
        cur = X.contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for Lr, W, b, s in zip(self.layers, self.W, self.b, self.s):
            out = torch.empty(cur.shape[0], Lr.out_dim, device=self.device, dtype=torch.float32)
            L.call("dgx_dense_q", cur.data_ptr(), W.data_ptr(), float(Lr.scale) if s is None else 0.0,
                   None if s is None else s.data_ptr(), b.data_ptr(), out.data_ptr(), cur.shape[0], Lr.out_dim,
                   Lr.in_dim, int(Lr.relu), stream)
            cur = out
        return cur


# ---------------------------------------------------------------- per-channel exporter
def quantize_rows_per_channel(W: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """The exporter's per-tensor rule applied to each weight row: scale =
    max|w|/127 (1 if the row is ~0), q = clamp(round-half-away(clamp(w/scale,
    -128, 127)), -128, 127)."""
    W = np.asarray(W, np.float64)
    mx = np.abs(W).max(axis=1)
    scale = np.where(mx > 1e-30, mx / 127.0, 1.0)
    v = np.clip(W / scale[:, None], -128.0, 127.0)
    q = np.sign(v) * np.floor(np.abs(v) + 0.5)  # std::lround
    return np.clip(q, -128, 127).astype(np.int8), scale


def _c_float(v: float) -> str:
    s = "%.9g" % np.float32(v)
    if not any(c in s for c in ".eEni"):
        s += ".0"
    return s + "f"


def _c_name(name: str) -> str:
    out = re.sub(r"[^A-Za-z0-9_]", "_", name)
    return "_" + out if out[:1].isdigit() else out


def export_c_header_int8_per_channel(layers: Sequence[Tuple[str, np.ndarray, np.ndarray]], prefix: str,
                                     func_name: str = "predict") -> int:
    """Write prefix.h / prefix.c in the int8 exporter's layout with one
    scale per output channel. `layers`: (name, W [out, in], bias [out]) in
    network order; ReLU after every layer but the last. Returns the bytes of
    int8 weights + float32 scales and biases."""
    layers = [(n, np.asarray(W, np.float64), np.asarray(b, np.float64).reshape(-1)) for n, W, b in layers]
    if not layers:
        raise ValueError("no layers")
    base = os.path.basename(prefix)
    up = _c_name(base).upper()
    in_dim, out_dim = layers[0][1].shape[1], layers[-1][1].shape[0]
    max_buf = max(W.shape[0] for _, W, _ in layers)
    d = os.path.dirname(prefix)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(prefix + ".h", "w") as f:
        f.write(f"/*\n * {base}.h - int8 quantized, one scale per output channel\n *\n"
                f" * Input dim: {in_dim}, Output dim: {out_dim}, Layers: {len(layers)}\n"
                f" * Quantization: per-channel symmetric, weights only (activations stay float).\n */\n"
                f"#ifndef {up}_H\n#define {up}_H\n\n#include <stdint.h>\n\n"
                f"#ifdef __cplusplus\nextern \"C\" {{\n#endif\n\n"
                f"#define {up}_INPUT_DIM  {in_dim}\n#define {up}_OUTPUT_DIM {out_dim}\n"
                f"#define {up}_NUM_LAYERS {len(layers)}\n#define {up}_QUANTIZED  2\n\n"
                f"void {func_name}(const float* input, float* output);\n\n"
                f"#ifdef __cplusplus\n}}\n#endif\n\n#endif /* {up}_H */\n")
    nbytes = 0
    with open(prefix + ".c", "w") as f:
        f.write(f"/* {base}.c - int8 quantized, one scale per output channel */\n"
                f"#include \"{base}.h\"\n#include <stdint.h>\n#include <math.h>\n\n")
        names = []
        for name, W, b in layers:
            q, sc = quantize_rows_per_channel(W)
            wn, bn = _c_name(name + ".weight"), _c_name(name + ".bias")
            names.append((wn, bn, W.shape[0]))
            f.write(f"/* {name}.weight shape: [{W.shape[0]}, {W.shape[1]}], quantized int8, per channel */\n")
            f.write(f"static const int8_t {wn}[{q.size}] = {{")
            flat = q.reshape(-1)
            for i, v in enumerate(flat):
                f.write(("\n    " if i % 16 == 0 else "") + str(int(v)) + (", " if i + 1 < flat.size else ""))
            f.write("\n};\n")
            f.write(f"static const float {wn}_scale[{sc.size}] = {{")
            for i, v in enumerate(sc):
                f.write(("\n    " if i % 8 == 0 else "") + _c_float(v) + (", " if i + 1 < sc.size else ""))
            f.write("\n};\n\n")
            f.write(f"/* {name}.bias shape: [{b.size}], float32 */\n")
            f.write(f"static const float {bn}[{b.size}] = {{")
            for i, v in enumerate(b):
                f.write(("\n    " if i % 8 == 0 else "") + _c_float(v) + (", " if i + 1 < b.size else ""))
            f.write("\n};\n\n")
            nbytes += q.size + 4 * sc.size + 4 * b.size
        f.write("/* Dense layer with int8 weights and one scale per output channel. */\n"
                "/* y[j] = bias[j] + scale[j] * sum_k (int8_w[j*in + k] * x[k]) */\n"
                "static void dense_qc(const float* x, int in_dim,\n"
                "                     const int8_t* w, const float* scale, const float* b,\n"
                "                     float* y, int out_dim) {\n"
                "    for (int j = 0; j < out_dim; ++j) {\n"
                "        float acc = b[j];\n"
                "        const int8_t* wr = w + j * in_dim;\n"
                "        for (int k = 0; k < in_dim; ++k) {\n"
                "            acc += scale[j] * ((float)wr[k]) * x[k];\n"
                "        }\n"
                "        y[j] = acc;\n"
                "    }\n"
                "}\n\n"
                "static void relu_inplace(float* x, int n) {\n"
                "    for (int i = 0; i < n; ++i) if (x[i] < 0.0f) x[i] = 0.0f;\n"
                "}\n\n")
        f.write(f"void {func_name}(const float* input, float* output) {{\n"
                f"    float buf_a[{max_buf}];\n    float buf_b[{max_buf}];\n"
                f"    const float* cur_in = input;\n    int cur_dim = {up}_INPUT_DIM;\n"
                f"    float* cur_out;\n    int use_a = 1;\n\n")
        for i, (wn, bn, out) in enumerate(names):
            if i == len(names) - 1:
                f.write(f"    /* layer {i} -> output */\n"
                        f"    dense_qc(cur_in, cur_dim, {wn}, {wn}_scale, {bn}, output, {out});\n")
            else:
                f.write(f"    /* layer {i} */\n    cur_out = use_a ? buf_a : buf_b;\n"
                        f"    dense_qc(cur_in, cur_dim, {wn}, {wn}_scale, {bn}, cur_out, {out});\n"
                        f"    relu_inplace(cur_out, {out});\n    cur_in = cur_out;\n    cur_dim = {out};\n"
                        f"    use_a = !use_a;\n\n")
        f.write("}\n")
    return nbytes
