"""The allocation-free entry point (blackhole_sm100_nvfp4_bf16_gemm_noalloc), called through
the C ABI.

This path exists for callers that may not allocate device memory when they run the GEMM:
serving engines that reserve their memory up front and forbid allocation afterwards, paths
that must not pay cudaMalloc's implicit synchronisation, and plugin hosts that hand a plugin
only its input and output buffers.  Its scratch is a fixed array inside the library that
every call reuses, so each case makes two calls in a row, the second starting from whatever
the first left behind, and checks both against the host oracle (parity tolerance) and bit for
bit against the regular entry point, which runs the same skinny schedule with a workspace of
its own.  The device's free memory must not move across the calls.  The file name makes pytest
collect it last."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(16, 4096, 2048), (1, 28672, 1024), (7, 1152, 4096)])
def test_noalloc_matches_oracle_and_regular_entry_point_twice(M, N, K):
    import torch
    import blackhole_b200 as bh

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=100 + M, std_b=0.02)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    regular = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, regular, alpha)
    torch.cuda.synchronize()
    regular_bits = regular.view(torch.int16).cpu().numpy().view(np.uint16)
    ref, absdot = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    free = []
    for out in outs:
        out.fill_(float("nan"))
        bh.nvfp4_bf16_gemm_noalloc(M, N, K, tA, tSFA, tB, tSFB, out, alpha)
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info(dev)[0])
        got_bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
        bad, maxerr, ratio, _ = O.check(ref, got_bits, alpha, K, absdot)
        assert bad == 0, f"{bad} elements outside tolerance (max err {maxerr}, err/tol {ratio})"
        assert np.array_equal(got_bits, regular_bits), "differs from the regular entry point"
    # the first call may have made the module's arrays resident; the second allocates nothing
    assert free[1] == free[0], f"free device memory moved by {free[0] - free[1]} bytes"
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
