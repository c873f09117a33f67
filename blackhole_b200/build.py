"""Builds the sm_100a CUDA library in-tree: blackhole_b200/libblackhole_sm100.so.

nvcc cross-compiles for sm_100a without a GPU.  The library is self-contained (static
cudart) and exports only the C ABI declared in include/blackhole_sm100.h.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libblackhole_sm100.so")
SOURCES = [os.path.join(HERE, "csrc", "blackhole_sm100_capi.cu")]
HEADERS_DIR = os.path.join(ROOT, "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-v",
    "--expt-relaxed-constexpr",
    "-shared",
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _deps():
    out = list(SOURCES)
    for d, _, files in os.walk(HEADERS_DIR):
        out += [os.path.join(d, f) for f in files if f.endswith((".h", ".hpp", ".cuh"))]
    return out


def is_stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not is_stale():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", HEADERS_DIR, *SOURCES, "-o", LIB + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libblackhole_sm100.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
