#!/usr/bin/env bash
# Build the Dream runtime with the B200 backend: heellowdsf/DreamCompiler's
# runtime/ compiled from its own sources, with this directory's b200.inc
# included after backend/gpu.inc and one hook per hot branch, linked against
# libdgx. Output: dreamcompiler_b200/refside/libdream_ref_b200.so, a drop-in
# for the reference's libdream (same extern "C" ops on the same struct
# Tensor), whose tensor_matmul, dream_linear, dream_flash_attention and
# matching backward branches run on the B200.
#
#   bash dreamcompiler_b200/refside/build.sh <path to the DreamCompiler checkout>
#
# The reference sources are copied to a temporary directory and edited there
# (nothing of them is written into this repository):
#   runtime.h            the materialize declaration gets C linkage, as
#                        core/tensor.inc defines it inside extern "C" (g++
#                        rejects the mismatch otherwise)
#   runtime.cpp          #include "backend/b200.inc" after backend/gpu.inc
#   ops/elementwise.inc  tensor_matmul, dream_linear: return b200's result
#   nn/training.inc      dream_flash_attention: return b200's result
#   ops/autograd.inc     "matmul", "linear"/"linear_relu", "flash_attention":
#                        a preceding branch of the same test runs b200's
#                        backward, so the reference's branch body is skipped
#                        and the code after the branch chain still runs
# Compiler flags are the ones `dream run` uses (src/main.cpp:994) plus -fPIC.
set -euo pipefail
REF=${1:?usage: build.sh <DreamCompiler checkout>}
HERE="$(cd "$(dirname "$0")" && pwd)"
PKG="$(dirname "$HERE")"
ROOT="$(dirname "$PKG")"
[ -d "$REF/runtime" ] || { echo "runtime/ not found under $REF" >&2; exit 2; }
[ -f "$PKG/libdgx.so" ] || { echo "build libdgx.so first (python -m dreamcompiler_b200.build)" >&2; exit 2; }
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$REF/runtime" "$TMP/runtime"
cp "$HERE/b200.inc" "$TMP/runtime/backend/b200.inc"
python3 - "$TMP/runtime" <<'PY'
import sys
rt = sys.argv[1]

def edit(path, old, new):
    p = f"{rt}/{path}"
    s = open(p).read()
    if s.count(old) != 1:
        sys.exit(f"{path}: expected exactly one occurrence of {old!r}, found {s.count(old)}")
    open(p, "w").write(s.replace(old, new))

edit("runtime.h", "\nstatic inline Tensor* materialize(Tensor* t);\n",
     '\nextern "C" { static inline Tensor* materialize(Tensor* t); }\n')
edit("runtime.cpp", '#include "backend/gpu.inc"\n', '#include "backend/gpu.inc"\n#include "backend/b200.inc"\n')
edit("ops/elementwise.inc", "    int M=a->d0, K=a->d1, N=b->d1;\n",
     "    int M=a->d0, K=a->d1, N=b->d1;\n"
     "    if (Tensor* r_b200 = b200::matmul(a, b, c, M, K, N, g_autograd_enabled)) return r_b200;\n")
edit("ops/elementwise.inc", "    par[0] = x; par[1] = W; par[2] = b;\n    tensor_set_parents(out, par, 3);\n",
     "    par[0] = x; par[1] = W; par[2] = b;\n    tensor_set_parents(out, par, 3);\n"
     "    if (Tensor* r_b200 = b200::linear(x, W, b, out, N, in_dim, out_dim)) return r_b200;\n")
edit("nn/training.inc",
     '    out->bwd_name = std::to_string(B) + "," + std::to_string(S) + "," + std::to_string(dk);\n\n'
     '    std::vector<double> sc((size_t)Bc);',
     '    out->bwd_name = std::to_string(B) + "," + std::to_string(S) + "," + std::to_string(dk);\n'
     "    if (Tensor* r_b200 = b200::flash_forward(Q, K, V, out, B, S, dk)) return r_b200;\n\n"
     '    std::vector<double> sc((size_t)Bc);')
edit("ops/autograd.inc", '        } else if (fn=="matmul") {\n',
     '        } else if (fn=="matmul" && b200::matmul_backward(t)) {\n        } else if (fn=="matmul") {\n')
edit("ops/autograd.inc", '        } else if (fn=="linear" || fn=="linear_relu") {\n',
     '        } else if ((fn=="linear" || fn=="linear_relu") && b200::linear_backward(t)) {\n'
     '        } else if (fn=="linear" || fn=="linear_relu") {\n')
edit("ops/autograd.inc", '        } else if (fn=="flash_attention") {\n',
     '        } else if (fn=="flash_attention" && b200::flash_backward(t)) {\n'
     '        } else if (fn=="flash_attention") {\n')
PY
g++ -std=c++17 -O3 -ffast-math -mavx2 -mfma -fno-math-errno -DNDEBUG -fopenmp -fPIC -w \
    -I"$REF/src" -I"$ROOT/include" -DDREAM_NO_MAIN -shared "$TMP/runtime/runtime.cpp" \
    -o "$HERE/libdream_ref_b200.so" -L"$PKG" -ldgx \
    -Wl,-rpath,'$ORIGIN/..' -ldl
echo "built $HERE/libdream_ref_b200.so"
