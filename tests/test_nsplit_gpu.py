"""N-split on one GPU: every shard of B run through the C ABI as its own GEMM; the slices
placed side by side must equal the unsplit GEMM -- bit for bit on the tiled schedule (each
output tile sums K in the same order whatever the split), within the parity tolerance on
the skinny schedule (its stream-K split points move with N)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,world", [(256, 2048, 1024, 2), (384, 4096, 512, 4), (1024, 2048, 2048, 8),
                                         (16, 4096, 2048, 2), (1, 8192, 1024, 8)])
def test_shards_reassemble_to_full_gemm(M, N, K, world):
    import torch
    import blackhole_b200 as bh
    from blackhole_b200 import nsplit

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M + world, std_b=0.02)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    full = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, full, alpha)
    slices = [nsplit.nsplit_gemm(M, N, K, tA, tSFA, tB, tSFB, alpha, r, world) for r in range(world)]
    torch.cuda.synchronize()
    joined = torch.cat(slices, dim=1).view(torch.int16).cpu().numpy().view(np.uint16)
    ref = full.view(torch.int16).cpu().numpy().view(np.uint16)
    if M > 128:
        assert np.array_equal(joined, ref)
    else:
        _, absdot = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
        bad, *_ = O.check(ref, joined, alpha, K, absdot)
        assert bad == 0
    assert bh.device_status(0) == 0
