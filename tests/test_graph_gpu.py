"""CUDA graph capture and replay of the GEMM, as a serving engine runs it: each schedule is
captured once (after one eager call on the same stream, which sets up the library's
per-stream workspace and kernel attributes, so the capture allocates nothing) and replayed back
to back on that stream with new inputs copied into the captured buffers.  Every replay must
match the oracle on its inputs.  For the skinny schedule this checks that the launch tags kept
in the workspace advance on the device with every replay (the graph freezes the kernel
arguments), so no replay consumes an earlier replay's partial sums."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(16, 4096, 2048), (5, 1152, 4352), (128, 1024, 1024),
                                   (512, 1024, 1024)])
def test_graph_replays_match_the_oracle(M, N, K):
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    cases = [C.make_operands(M, N, K, seed=300 + 7 * i + M, std_b=0.02) for i in range(3)]
    alpha = cases[0][4]   # a captured kernel argument: the same for every replay
    bufs = [torch.from_numpy(x).to(dev) for x in cases[0][:4]]
    tA, tSFA, tB, tSFB = bufs
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha)
    srcs = [[torch.from_numpy(x).to(dev) for x in c[:4]] for c in cases]
    outs = []
    with torch.cuda.stream(s):
        for rep in range(2):
            for src in srcs:
                for dst, x in zip(bufs, src):
                    dst.copy_(x)
                D.fill_(float("nan"))
                g.replay()
                outs.append(D.view(torch.int16).clone())
    s.synchronize()
    assert bh.device_status(0) == 0
    for i, out in enumerate(outs):
        A, SFA, B, SFB, _ = cases[i % len(cases)]
        ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
        got = out.cpu().numpy().view(np.uint16)
        bad, maxerr, ratio, _ = O.check(ref, got, alpha, K, ad)
        assert bad == 0, f"replay {i}: {bad} elements outside tolerance (err/tol {ratio})"
        assert np.array_equal(got, outs[i % len(cases)].cpu().numpy().view(np.uint16))
    del g
