"""Builds the example and the library with the repository's CMakeLists.txt (the sm_100a
target a C++ user builds) into a scratch directory.  Used by the CPU build test and the GPU
example test."""
from __future__ import annotations

import os
import shutil
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def cmake_build(build_dir: str) -> dict:
    """Configures and builds every target; returns the paths of the built files."""
    cmake = shutil.which("cmake")
    if cmake is None:
        raise RuntimeError("cmake is not installed")
    gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    subprocess.run([cmake, "-S", ROOT, "-B", build_dir, *gen, "-DCMAKE_BUILD_TYPE=Release"],
                   check=True, capture_output=True, text=True)
    res = subprocess.run([cmake, "--build", build_dir, "-j", str(os.cpu_count() or 2)],
                         capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("cmake build failed:\n" + res.stdout[-4000:] + res.stderr[-4000:])
    return {name: os.path.join(build_dir, name)
            for name in ("libblackhole_sm100.so", "nvfp4_bf16_gemm_sm100", "nvfp4_bf16_gemm_capi")}
