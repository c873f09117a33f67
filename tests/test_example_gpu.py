"""The B200 example (example/nvfp4_bf16_gemm.cu), the reference example's counterpart, built
with the repository's CMake target and run: through the header-only operator (nvcc) and through
the C ABI (host compiler).  Each run makes the reference's nine-argument call, checks sampled
elements against the host loop (rel <= 0.05 and bit-identical, the inputs being exact), times
the GEMM and must exit 0."""
import os
import re
import subprocess

import pytest

from tests.example_build import cmake_build

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def built(tmp_path_factory):
    return cmake_build(str(tmp_path_factory.mktemp("example") / "build"))


@pytest.mark.parametrize("exe,args", [
    ("nvfp4_bf16_gemm_sm100", []),                                   # 4096^3, the default
    ("nvfp4_bf16_gemm_sm100", ["16", "4096", "4096", "--iters", "20"]),   # decode (skinny)
    ("nvfp4_bf16_gemm_sm100", ["200", "136", "544", "--iters", "5"]),     # ragged
    ("nvfp4_bf16_gemm_capi", ["2048", "2048", "2048", "--iters", "20"]),
    ("nvfp4_bf16_gemm_capi", ["1", "1024", "8192", "--iters", "20"]),
])
def test_example_runs_and_passes(built, exe, args):
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = os.path.dirname(built[exe]) + ":" + env.get("LD_LIBRARY_PATH", "")
    res = subprocess.run([built[exe], *args], capture_output=True, text=True, timeout=600, env=env)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "PASSED" in res.stdout
    m = re.search(r"Checked (\d+) elements: max_rel=([\d.]+), mismatches=(\d+), bit-identical=(\d+)",
                  res.stdout)
    assert m and m.group(1) == m.group(4) and m.group(3) == "0"
    assert re.search(r"Avg [\d.]+ ms\s+[\d.]+ TFLOP/s", res.stdout)
