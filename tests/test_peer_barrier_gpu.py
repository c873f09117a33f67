"""The gathered N-split's cross-GPU flag barrier (blackhole_sm100_peer_barrier) on one GPU.

A two-rank barrier is run for rank 0 with both ranks' flag arrays in local memory.  No launch
waits on another: either the peer's signal is already in place (the barrier must store its
own signal into the peer's array and return at once), or nothing ever sets it (the bounded
wait must give up after its short limit, set status bit 8 and return, leaving the context
usable).  The real two-GPU exchange runs in test_gather_multigpu.py."""
import time

import pytest

pytestmark = pytest.mark.gpu


def test_single_rank_is_a_no_op():
    import torch
    import blackhole_b200 as bh

    f = torch.zeros(1, dtype=torch.int64, device="cuda:0")
    bh.peer_barrier([f], 1, 0, 1)
    torch.cuda.synchronize()
    assert int(f.item()) == 0 and bh.device_status(0) == 0


def test_signals_the_peer_and_passes_when_the_peer_has_signalled():
    import torch
    import blackhole_b200 as bh

    bh.device_status(0, clear=True)
    own = torch.zeros(2, dtype=torch.int64, device="cuda:0")
    peer = torch.zeros(2, dtype=torch.int64, device="cuda:0")
    for epoch in (1, 2, 3):
        own[1] = epoch                      # rank 1's signal, already delivered
        bh.peer_barrier([own, peer], 2, 0, epoch, 1_000_000_000)
        torch.cuda.synchronize()
        assert int(peer[0].item()) == epoch  # this rank's signal in rank 1's array
        assert int(peer[1].item()) == 0 and int(own[0].item()) == 0
    assert bh.device_status(0) == 0


def test_missing_peer_times_out_with_status_and_context_stays_usable():
    import torch
    import blackhole_b200 as bh
    from tests import nvfp4_cases as C

    bh.device_status(0, clear=True)
    own = torch.zeros(2, dtype=torch.int64, device="cuda:0")
    peer = torch.zeros(2, dtype=torch.int64, device="cuda:0")
    t0 = time.perf_counter()
    bh.peer_barrier([own, peer], 2, 0, 1, 20_000_000)     # 20 ms; rank 1 never signals
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert bh.device_status(0, clear=True) == 8
    assert int(peer[0].item()) == 1
    M, N, K = 16, 1024, 1024
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=3)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, _, _, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0
