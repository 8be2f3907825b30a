"""Build recipe for the in-tree native libraries.

* ``libdgx.so``   — the sm_100a CUDA kernels behind the C ABI of include/dgx.h
* ``libdream_b200.so`` — the C++ Dream-runtime mirror (Tensor, tensor_matmul,
  dream_flash_attention, backward, ...) that forwards into libdgx

Both land next to this file so they travel with the source tree. Objects are
rebuilt only when a source or header is newer than the library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
RTSRC = os.path.join(HERE, "runtime")
BUILD = os.path.join(ROOT, "_build")
LIBDGX = os.path.join(HERE, "libdgx.so")
LIBRT = os.path.join(HERE, "libdream_b200.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + os.path.basename(cmd[-1]))


def build_libdgx(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                     + glob.glob(os.path.join(ROOT, "include", "*.h")))
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        if _newer(o, [s] + headers) or ptxas_verbose:
            cmd = [NVCC] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError("nvcc failed on " + os.path.basename(s))
            if ptxas_verbose:
                sys.stdout.write(r.stderr)
        objs.append(o)
    if _newer(LIBDGX, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIBDGX] + objs
             + ["-cudart", "shared", "-Xlinker", "-rpath," + os.path.join(CUDA_HOME, "lib64"), "-ldl"])
    return LIBDGX


# Flags `dream run` compiles the reference runtime with (src/main.cpp:994);
# used for the runtime files that must reproduce its floating-point results
# bit for bit (the seeded RNG), named *_fastmath.cpp.
REF_FLAGS = ["-O3", "-ffast-math", "-mavx2", "-mfma", "-fno-math-errno"]


def build_runtime(verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(RTSRC, "*.cpp")))
    if not srcs:
        return ""
    deps = srcs + sorted(glob.glob(os.path.join(RTSRC, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h")))
    if _newer(LIBRT, deps + [LIBDGX]):
        os.makedirs(BUILD, exist_ok=True)
        objs = []
        for s in srcs:
            o = os.path.join(BUILD, os.path.basename(s) + ".o")
            flags = REF_FLAGS if s.endswith("_fastmath.cpp") else ["-O2"]
            cmd = ["g++", "-std=c++17", "-fPIC", "-Wall", "-I" + os.path.join(ROOT, "include"),
                   "-I" + os.path.join(CUDA_HOME, "include")] + flags + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
            objs.append(o)
        _run(["g++", "-shared", "-o", LIBRT] + objs + [
            "-L" + HERE, "-ldgx", "-Wl,-rpath,$ORIGIN",
            "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")])
    return LIBRT


def build_all(verbose: bool = False) -> None:
    if not shutil.which(NVCC) and not os.path.exists(NVCC):
        raise RuntimeError("nvcc not found at " + NVCC)
    build_libdgx(verbose)
    build_runtime(verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    if "--ptxas" in sys.argv:
        build_libdgx(ptxas_verbose=True)
