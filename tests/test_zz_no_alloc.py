"""The allocation-free entry point (blackhole_sm100_nvfp4_bf16_gemm_noalloc), called through
the C ABI and checked against the regular entry point on the same inputs.

This path exists for callers that may not allocate device memory when they run the GEMM
(memory planned up front, no cudaMalloc synchronisation allowed on the path, hosts that
pass only inputs and outputs).  Its scratch is a fixed array inside the library that every
call reuses, so the test makes two calls in a row: the second one starts from whatever the
first left behind.  The file name makes pytest collect it last."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(16, 4096, 2048), (1, 28672, 1024), (7, 1152, 4096)])
def test_noalloc_matches_regular_entry_point_twice(M, N, K):
    import torch
    import blackhole_b200 as bh

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=100 + M, std_b=0.02)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, ref, alpha)
    torch.cuda.synchronize()
    ref_bits = ref.view(torch.int16).cpu().numpy().view(np.uint16)
    # per-element tolerance of the parity tests: one BF16 ulp + FP32 reassociation slack
    _, absdot = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        bh.nvfp4_bf16_gemm_noalloc(M, N, K, tA, tSFA, tB, tSFB, out, alpha)
        torch.cuda.synchronize()
        got_bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
        bad, maxerr, ratio, _ = O.check(ref_bits, got_bits, alpha, K, absdot)
        assert bad == 0, f"{bad} elements differ beyond tolerance (max err {maxerr}, err/tol {ratio})"
    assert bh.device_status(0) == 0


def test_noalloc_rejects_m_beyond_its_array():
    import torch
    import blackhole_b200 as bh

    M, N, K = 17, 128, 256
    dev = torch.device("cuda:0")
    A = torch.zeros(M * K // 2, dtype=torch.uint8, device=dev)
    B = torch.zeros(N * K // 2, dtype=torch.uint8, device=dev)
    SF = torch.zeros(bh.sf_storage_bytes(128, K), dtype=torch.uint8, device=dev)
    D = torch.zeros((M, N), dtype=torch.bfloat16, device=dev)
    with pytest.raises(bh.BlackholeError) as ei:
        bh.nvfp4_bf16_gemm_noalloc(M, N, K, A, SF, B, SF, D)
    assert ei.value.code == 1  # cudaErrorInvalidValue
