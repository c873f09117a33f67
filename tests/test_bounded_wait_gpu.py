"""The bounded-wait / abort protocol of the GEMM kernels, exercised on the GPU without a fault.

The skinny schedule's recovery is exercised the same way: a launch whose finishers give up
on a 1 ns wait for partial sums (self-test hook), then a normal launch on the same workspace.

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


def _device_operands(M, N, K, seed):
    import torch
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=seed, std_b=0.02)
    dev = torch.device("cuda:0")
    return (A, SFA, B, SFB, alpha), [torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB)]


def test_skinny_workspace_recovers_after_an_aborted_launch():
    """A skinny launch whose finishing CTAs give up waiting for partial sums (a 1 ns bound
    through the self-test hook) leaves flags of its workspace raised.  The next launch on the
    same workspace, with other inputs, must not take those flags for its own: its result matches
    the oracle and a launch on a fresh workspace bit for bit."""
    import numpy as np
    import torch
    import blackhole_b200 as bh

    M, N, K = 16, 8192, 8192
    dev = torch.device("cuda:0")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ws = torch.zeros(bh.workspace_bytes(M, N, K), dtype=torch.uint8, device=dev)
    words = ws.view(torch.int32)
    (_, _, _, _, alpha1), t1 = _device_operands(M, N, K, 1)
    (A, SFA, B, SFB, alpha2), t2 = _device_operands(M, N, K, 2)
    bh.device_status(0, clear=True)
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    launches, raised = 0, 0
    for _ in range(5):
        bh.selftest_skinny_partial_wait(M, N, K, *t1, D, alpha1, ws, 1)
        launches += 1
        status = bh.device_status(0, clear=True)
        assert (status & ~4) == 0, f"status {status:#x}: only the epilogue (bit 2) may give up"
        raised = int(torch.count_nonzero(words[:8 * sms]).item())
        if status & 4 and raised:
            break
    assert status & 4 and raised, "no finisher gave up: the scenario did not occur"
    assert int(words[8 * sms].item()) == 0, "ticket counter not reset by the aborted launch"
    assert int(words[8 * sms + 1].item()) == launches, "launch generation not advanced"
    # the next launch on the same workspace, with other inputs
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    bh.nvfp4_bf16_gemm_ex(M, N, K, *t2, out, alpha2, schedule="skinny", workspace=ws)
    fresh = torch.zeros_like(ws)
    out_fresh = torch.empty_like(out)
    bh.nvfp4_bf16_gemm_ex(M, N, K, *t2, out_fresh, alpha2, schedule="skinny", workspace=fresh)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    (bad, maxerr, ratio, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha2, got)
    assert bad == 0, f"{bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"
    assert np.array_equal(got, out_fresh.view(torch.int16).cpu().numpy().view(np.uint16))
    assert int(words[8 * sms].item()) == 0 and int(words[8 * sms + 1].item()) == launches + 1


def test_skinny_partial_wait_bound_out_of_range_rejected():
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    t = [torch.zeros(1 << 20, dtype=torch.uint8, device=dev) for _ in range(4)]
    D = torch.zeros((16, 128), dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(bh.workspace_bytes(16, 128, 256), dtype=torch.uint8, device=dev)
    for bound in (0, 5_000_000_000):
        with pytest.raises(bh.BlackholeError):
            bh.selftest_skinny_partial_wait(16, 128, 256, *t, D, 1.0, ws, bound)
