"""The one-SM schedule split stream-K over every SM (schedule "1sm_streamk"), against the CPU
oracle through the C ABI.

Cases cover a tile split over many CTAs (4 tiles of 32 k-tiles on 128 CTAs: each finisher adds
31 partials), decode widths with fewer tiles than SMs, ragged M / N and a K tail, a single
unit, and repeat determinism (the partials are added in a fixed order)."""
import numpy as np
import pytest

from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [
    (256, 512, 8192),     # 4 tiles x 32 k-tiles = 128 units: every tile split over 32 CTAs
    (128, 4096, 2048),    # 16 tiles x 8 k-tiles over 128 CTAs
    (100, 1000, 1056),    # ragged M and N, K tail (sf_tail maps)
    (17, 256, 256),       # one unit, one CTA
    (64, 2048, 4096),
    (200, 3072, 512),     # two tile-rows
])
def test_streamk_full(M, N, K):
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M + N, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule="1sm_streamk")
    (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


@pytest.mark.parametrize("M", [32, 64, 128])
def test_streamk_config2_decode_sampled(M):
    N, K = 28672, 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=2, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule="1sm_streamk")
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    assert not np.any(got == 0xFFFF), "unwritten output elements"


def test_streamk_deterministic_and_workspace_reusable():
    M, N, K = 256, 512, 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=77)
    outs = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, repeat=3, schedule="1sm_streamk")
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
