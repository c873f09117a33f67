"""The CMake sm_100a target builds on a machine without a GPU: the C-ABI library (exporting
every symbol include/*.h declares), the example through the header-only operator (nvcc) and
the same example through the C ABI (host compiler only).  Running them is tests/test_example_gpu.py."""
import os
import subprocess

from tests.example_build import cmake_build
from tests.test_capi_cpu import declared_symbols


def test_cmake_builds_library_and_both_examples(tmp_path):
    out = cmake_build(str(tmp_path / "build"))
    for path in out.values():
        assert os.path.isfile(path), path
    nm = subprocess.run(["nm", "-D", "--defined-only", out["libblackhole_sm100.so"]],
                        capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in nm.splitlines() if " T " in l}
    assert declared_symbols() <= exported
    # the C-ABI example needs no device code of its own: it links the library
    ldd = subprocess.run(["ldd", out["nvfp4_bf16_gemm_capi"]], capture_output=True, text=True).stdout
    assert "libblackhole_sm100.so" in ldd
