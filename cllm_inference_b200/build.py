"""Build the in-tree native libraries of cllm_inference_b200.

* lib/libcllm_cuda.so   — the CUDA kernels and the C ABI (include/cllm_cuda.h),
                           compiled for sm_100a only.
* lib/libcllm_quant.so  — the C++20 drop-in for the reference's quant.hpp API
                           (csrc/shim), linked against libcllm_cuda.so.
* lib/quant_shim_test   — a C++ test driver for the shim (run by tests/).

nvcc cross-compiles without a GPU, so this runs on the CPU build host too.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))
CUDA_INC = os.path.join(CUDA_HOME, "include")
CUDA_LIBDIR = os.path.join(CUDA_HOME, "lib64")

CUDA_SO = os.path.join(LIB, "libcllm_cuda.so")
SHIM_SO = os.path.join(LIB, "libcllm_quant.so")
SHIM_TEST = os.path.join(LIB, "quant_shim_test")


def _sources(*dirs):
    out = []
    for d in dirs:
        for f in sorted(os.listdir(d)):
            if f.endswith((".cu", ".cuh", ".h", ".hpp", ".cpp")):
                out.append(os.path.join(d, f))
    return out


def _digest(deps):
    h = hashlib.sha256()
    for d in sorted(deps):
        h.update(os.path.relpath(d, ROOT).encode())  # the repository may live elsewhere on another machine
        with open(d, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _stale(target, deps):
    """A target is stale unless it exists and was built from exactly these
    sources (a digest of their contents is kept beside it), so an edit made
    while a build runs is never mistaken for built."""
    stamp = target + ".sources"
    if not os.path.exists(target) or not os.path.exists(stamp):
        return True
    with open(stamp) as f:
        return f.read().strip() != _digest(deps)


def _mark(target, deps, digest):
    with open(target + ".sources", "w") as f:
        f.write(digest)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> None:
    os.makedirs(LIB, exist_ok=True)
    deps = _sources(CSRC) + [os.path.join(INCLUDE, "cllm_cuda.h")]
    if force or ptxas_info or _stale(CUDA_SO, deps):
        digest = _digest(deps)  # of the sources as compiled
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
               "-o", CUDA_SO, os.path.join(CSRC, "cllm_cuda.cu")]
        if ptxas_info:
            cmd[1:1] = ["-Xptxas", "-v"]
        _run(cmd, verbose)
        _mark(CUDA_SO, deps, digest)
    shim_dir = os.path.join(CSRC, "shim")
    shim_deps = _sources(shim_dir, os.path.join(shim_dir, "cllm", "core")) + [CUDA_SO]
    if os.path.exists(os.path.join(shim_dir, "quant_shim.cpp")):
        if force or _stale(SHIM_SO, shim_deps):
            shim_digest = _digest(shim_deps)
            _run(["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-fPIC", "-shared",
                  "-I", shim_dir, "-I", INCLUDE, "-I", CUDA_INC, "-o", SHIM_SO,
                  os.path.join(shim_dir, "quant_shim.cpp"), "-L", LIB, "-lcllm_cuda",
                  "-L", CUDA_LIBDIR, "-lcudart_static", "-ldl", "-lrt", "-pthread",
                  "-Wl,-rpath,$ORIGIN"], verbose)
            _mark(SHIM_SO, shim_deps, shim_digest)
        test_src = os.path.join(shim_dir, "quant_shim_test.cpp")
        test_deps = shim_deps + [SHIM_SO]
        if os.path.exists(test_src) and (force or _stale(SHIM_TEST, test_deps)):
            test_digest = _digest(test_deps)
            _run(["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-I", shim_dir, "-I", INCLUDE,
                  "-o", SHIM_TEST, test_src, "-L", LIB, "-lcllm_quant", "-lcllm_cuda",
                  "-Wl,-rpath,$ORIGIN"], verbose)
            _mark(SHIM_TEST, test_deps, test_digest)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
