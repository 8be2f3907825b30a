#!/usr/bin/env bash
# TEST INFRASTRUCTURE. Compiles the reference Dream runtime (heellowdsf/
# DreamCompiler, runtime/) from its own sources into oracle/_ref/libdream_ref.so
# so the tests can pin the CPU oracle against the reference itself and
# bench.py can time the reference's own CPU path.
#
# The sources are compiled where they lie except for one file: runtime.h:109
# declares `materialize` with C++ linkage and runtime.cpp then re-declares it
# inside an extern "C" block (core/tensor.inc:141), which g++ rejects. The
# script copies runtime/ to a temporary directory, wraps that one declaration
# in extern "C" there, and compiles the copy with the flags `dream run` uses
# (src/main.cpp:994) plus -fPIC. Nothing from the reference is written into
# this repository except the compiled library under oracle/_ref/.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
# The reference checkout sits beside this repository unless an argument names it.
REF=${1:-$(dirname "$(dirname "$HERE")")/reference}
OUT="$HERE/_ref"
[ -d "$REF/runtime" ] || { echo "reference runtime not found at $REF/runtime" >&2; exit 2; }
mkdir -p "$OUT"
TMP="$(mktemp -d)"
trap 'rm -rf "$TMP"' EXIT
cp -r "$REF/runtime" "$TMP/runtime"
sed -i 's/^static inline Tensor\* materialize(Tensor\* t);$/extern "C" { static inline Tensor* materialize(Tensor* t); }/' \
    "$TMP/runtime/runtime.h"
g++ -std=c++17 -O3 -ffast-math -mavx2 -mfma -fno-math-errno -DNDEBUG -fopenmp -fPIC -w \
    -I"$REF/src" -DDREAM_NO_MAIN -shared "$TMP/runtime/runtime.cpp" -o "$OUT/libdream_ref.so" -ldl
echo "built $OUT/libdream_ref.so"
