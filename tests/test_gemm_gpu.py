"""GPU parity of the sm_100a NVFP4 GEMM against the CPU oracle, through the C ABI.

Tolerance (per element): |got - ref| <= ulp_bf16(max(|ref|,|got|)) + |alpha|*K*2^-24*sum_k|a_k b_k|,
i.e. one BF16 ulp of the output plus the worst-case FP32 reassociation error of the K-term
sum; the per-term products are exact in FP32.  The reference example's own check
(rel <= 0.05, example/nvfp4_bf16_gemm.cu:169-172) is asserted as well."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _gold(name):
    man = json.load(open(os.path.join(GOLD, "manifest.json")))
    dt = {"uint8": np.uint8, "uint16": np.uint16}[man[name]["dtype"]]
    return np.fromfile(os.path.join(GOLD, name), dtype=dt)


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (256, 384, 512)])
def test_reference_example_fixtures_bit_exact(M, N, K):
    """Inputs drawn like the reference example; every partial sum is exact in FP32, so the
    GPU must reproduce the example's host loop bit for bit."""
    p = f"gemm_{M}x{N}x{K}_"
    A, SFA, B, SFB, D = (_gold(p + s) for s in ("A.u8", "SFA.u8", "B.u8", "SFB.u8", "D.u16"))
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, 1.0)
    assert np.array_equal(got.ravel(), D)


def test_config0_full_1024_cubed():
    M = N = K = 1024
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=0)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} elements outside tolerance (max err {maxerr}, max err/tol {ratio})"
    assert rel <= 0.05


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 256),      # one tile, one k-tile
    (128, 128, 512),      # N % 256 == 128: half of the B box is out of range
    (200, 384, 768),      # ragged M, ragged N tile, 3 k-tiles
    (1, 256, 1024),       # decode M=1
    (16, 1024, 2048),     # decode M=16
    (64, 512, 4096),
    (384, 640, 256),
    (130, 128, 8192),     # long K
])
def test_shapes_full(M, N, K):
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M * 7 + N, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


def test_alpha_scales_output():
    M, N, K = 128, 256, 512
    A, SFA, B, SFB, _ = C.make_operands(M, N, K, seed=11)
    for alpha in (1.0, 0.5, -3.25, 1e-3):
        got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
        (bad, *_), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
        assert bad == 0


def test_outlier_activations_config3_style():
    M, N, K = 256, 512, 2048
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=3, std_b=0.02, outlier_p=0.01)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, *_), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0


def test_deterministic_across_runs():
    M, N, K = 256, 512, 1024
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=5)
    outs = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, repeat=3)
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


@pytest.mark.parametrize("M", [1, 16, 64, 128])
def test_config2_decode_sampled(M):
    N, K = 28672, 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=2, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


def test_config1_8192_cubed_sampled():
    M = N = K = 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=1)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    assert rel <= 0.05
    assert not np.any(got == 0xFFFF), "unwritten output elements"
