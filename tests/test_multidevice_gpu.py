"""One process driving two GPUs: calls alternate between devices (the current device switched
between them), every schedule on each, from one host thread.  The library's set-up, workspaces,
kernel attributes and the thread's context binding are per device; the reference keeps a single
process-wide flag for its kernel attribute (nvfp4_gemm.hpp:625-631), which leaves every device
after the first without it.  Needs two GPUs (skipped otherwise)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu

SHAPES = [(16, 4096, 2048), (128, 1024, 1024), (512, 1024, 1024)]


def test_calls_alternate_between_two_devices():
    import torch
    import blackhole_b200 as bh

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    work = []
    for d in (0, 1):
        for M, N, K in SHAPES:
            c = C.make_operands(M, N, K, seed=600 + 13 * d + M, std_b=0.02)
            dev = torch.device(f"cuda:{d}")
            work.append((d, M, N, K, c, [torch.from_numpy(x).to(dev) for x in c[:4]],
                         torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)))
    for rep in range(3):
        for d, M, N, K, c, t, out in sorted(work, key=lambda w: (w[1], w[0])):
            with torch.cuda.device(d):
                bh.nvfp4_bf16_gemm(M, N, K, *t, out, c[4])
    for d in (0, 1):
        torch.cuda.synchronize(d)
        assert bh.device_status(d) == 0
    for d, M, N, K, c, _, out in work:
        A, SFA, B, SFB, alpha = c
        ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
        got = out.view(torch.int16).cpu().numpy().view(np.uint16)
        bad, maxerr, ratio, _ = O.check(ref, got, alpha, K, ad)
        assert bad == 0, f"device {d}, {M}x{N}x{K}: {bad} outside tolerance (err/tol {ratio})"
