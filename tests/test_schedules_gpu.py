"""Each GEMM schedule forced explicitly through the C ABI and checked element by element
against the oracle: the one-SM and two-SM tensor-core schedules on ragged shapes, and the
skinny-M stream-K schedule on shapes whose row blocks are split across many CTAs."""
import numpy as np
import pytest

from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


def _check(M, N, K, schedule, seed=0, std_b=1.0, workspace=None, repeat=1):
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=seed, std_b=std_b)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule=schedule, workspace=workspace,
                    repeat=repeat)
    outs = got if repeat > 1 else [got]
    for g in outs:
        (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, g)
        assert bad == 0, f"{schedule} {M}x{N}x{K}: {bad} bad (max err {maxerr}, err/tol {ratio})"
        assert not np.any(g == 0xFFFF)
    if repeat > 1:
        for g in outs[1:]:
            assert np.array_equal(g, outs[0]), "schedule is not deterministic"


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 768, 512), (384, 384, 1024),
                                   (200, 128, 256), (1000, 1152, 768), (2048, 2048, 2048),
                                   (256, 4096, 256)])
def test_two_sm_schedule(M, N, K):
    _check(M, N, K, "2sm", seed=M + N + K)


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 640, 512), (1024, 1024, 1024),
                                   (17, 512, 1024), (33, 1000, 512), (64, 4096, 2048),
                                   (100, 896, 4352), (48, 2048, 8192)])
def test_one_sm_schedule(M, N, K):
    _check(M, N, K, "1sm", seed=M + 3 * N + K)


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (5, 1024, 2048), (16, 4096, 8192),
                                   (17, 2048, 4096), (33, 1280, 1024), (64, 4096, 2048),
                                   (100, 896, 4352), (128, 4096, 8192), (16, 28672, 512)])
def test_skinny_schedule(M, N, K):
    _check(M, N, K, "skinny", seed=M * 11 + N, std_b=0.02, repeat=2)


def test_skinny_caller_workspace_reused_across_shapes():
    import torch
    import blackhole_b200 as bh
    need = max(bh.workspace_bytes(m, 4096, 4096) for m in (1, 16, 64, 128))
    assert need > 0 and bh.workspace_bytes(256, 4096, 4096) == 0
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for M in (16, 128, 1, 64, 16):
        _check(M, 2048, 4096, "skinny", seed=M, std_b=0.02, workspace=ws)
    # every call leaves the flag words (at the start of the workspace) zeroed
    torch.cuda.synchronize()
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    assert int(ws[: nsm * 16].count_nonzero()) == 0


def test_skinny_rejects_large_m_and_short_workspace():
    import torch
    import blackhole_b200 as bh
    A = torch.zeros(256 * 128, dtype=torch.uint8, device="cuda")
    SF = torch.zeros(bh.sf_storage_bytes(256, 256), dtype=torch.uint8, device="cuda")
    D = torch.zeros(256 * 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(bh.BlackholeError):
        bh.nvfp4_bf16_gemm_ex(256, 128, 256, A, SF, A, SF, D, schedule="skinny")
    small = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(bh.BlackholeError):
        bh.nvfp4_bf16_gemm_ex(16, 128, 256, A, SF, A, SF, D, schedule="skinny", workspace=small)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0


@pytest.mark.parametrize("schedule,M,N,K", [
    ("1sm", 256, 200, 512), ("1sm", 300, 1000, 768), ("2sm", 512, 136, 512),
    ("2sm", 640, 1304, 1024), ("skinny", 16, 1000, 2048), ("skinny", 7, 8, 256),
    ("skinny", 100, 2056, 1024), ("auto", 1024, 3000, 512)])
def test_ragged_n(schedule, M, N, K):
    """N not a multiple of 128 (only N % 8 == 0): B rows and SFB blocks past N read zeros, D
    columns past N are never written."""
    _check(M, N, K, schedule, seed=M + 7 * N + K)


@pytest.mark.parametrize("schedule,M,N,K", [
    ("1sm", 256, 512, 320), ("1sm", 300, 640, 1088), ("2sm", 512, 512, 576),
    ("2sm", 640, 768, 800), ("skinny", 16, 1024, 320), ("skinny", 5, 2048, 1056),
    ("skinny", 100, 512, 96), ("skinny", 1, 136, 32), ("auto", 1024, 1024, 2080),
    ("auto", 300, 1000, 1888)])
def test_k_tail(schedule, M, N, K):
    """K not a multiple of 256 (only K % 32 == 0): the last k-tile's A/B bytes past K and its
    scale-factor atoms past the last one read zeros."""
    _check(M, N, K, schedule, seed=3 * M + N + K)


@pytest.mark.parametrize("M", [16, 17, 64, 128, 256, 257])
def test_auto_schedule_matches_the_explicit_one(M):
    """By shape: M <= 16 skinny, M <= 256 one-SM, larger two-SM; bit-identical to that schedule
    forced explicitly."""
    N, K = 1024, 2048
    want = "skinny" if M <= 16 else ("1sm" if M <= 256 else "2sm")
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M)
    auto = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    forced = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule=want)
    assert np.array_equal(auto, forced)
    (bad, _, _, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, auto)
    assert bad == 0
