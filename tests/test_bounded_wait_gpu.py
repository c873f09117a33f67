"""The bounded-wait / abort protocol of the GEMM kernels, exercised on the GPU without a fault.

A self-test kernel plays a pipeline whose partner never arrives: its producer warp waits on
an mbarrier that nothing signals and gives up after a short limit, raising the CTA abort flag
and status bit 0; its consumer warp, which holds TMEM, must leave through the abort flag
(status bit 1 clear) and free its TMEM.  The test then checks that the context is still
usable: a GEMM on the same device (which allocates TMEM on every SM) matches the oracle."""
import time

import pytest

from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000  # 50 ms


def test_timeout_sets_status_and_kernel_returns():
    import torch
    import blackhole_b200 as bh

    bh.device_status(0, clear=True)
    result = torch.full((4,), -1, dtype=torch.int64, device="cuda:0")
    t0 = time.perf_counter()
    bh.selftest_bounded_wait(LIMIT_NS, result)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    status = bh.device_status(0, clear=True)
    done0, done1, wait0, wait1 = (int(v) for v in result.cpu())
    assert status == 1, f"status {status:#x}: expected the producer (bit 0) timeout only"
    assert (done0, done1) == (0, 0)
    assert LIMIT_NS <= wait0 < 20 * LIMIT_NS
    # the consumer leaves through the abort flag, long before its own 4x limit
    assert wait1 < 2 * LIMIT_NS
    assert wall < 5.0


def test_context_usable_after_timeout():
    import blackhole_b200 as bh
    import torch

    result = torch.zeros((4,), dtype=torch.int64, device="cuda:0")
    for _ in range(3):
        bh.selftest_bounded_wait(LIMIT_NS // 10, result)
    torch.cuda.synchronize()
    assert bh.device_status(0, clear=True) == 1
    M, N, K = 256, 1024, 2048
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=91)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)  # asserts the status is clean afterwards
    (bad, maxerr, ratio, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"


@pytest.mark.parametrize("limit", [0, 3_000_000_000])
def test_limit_out_of_range_rejected(limit):
    import torch
    import blackhole_b200 as bh

    result = torch.zeros((4,), dtype=torch.int64, device="cuda:0")
    with pytest.raises(bh.BlackholeError):
        bh.selftest_bounded_wait(limit, result)
