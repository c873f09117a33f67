"""GEMMs in flight on several streams at once, and from several host threads at once.

The library keeps one workspace per (device, stream) and per-thread tensor-map caches; the
skinny schedule's CTAs wait only on CTAs that started before them, so two of its launches on
different streams may share the GPU in any interleaving.  Every output must match the oracle
on its own inputs.  The threads test runs its threads twice: the second time every piece of
per-device set-up is already cached, so a new thread's first call does no set-up of its own."""
import threading

import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu

SHAPES = [(16, 4096, 2048), (128, 1024, 1024), (512, 1024, 1024)]


def _cases(M, N, K, n, base):
    return [C.make_operands(M, N, K, seed=base + 11 * i + M, std_b=0.02) for i in range(n)]


def _check(M, N, K, case, got_i16):
    A, SFA, B, SFB, alpha = case
    ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    got = got_i16.cpu().numpy().view(np.uint16)
    bad, maxerr, ratio, _ = O.check(ref, got, alpha, K, ad)
    assert bad == 0, f"{bad} elements outside tolerance (err/tol {ratio})"


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_launches_interleaved_on_two_streams(M, N, K):
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    cases = _cases(M, N, K, 4, 400)
    dev_cases = [[torch.from_numpy(x).to(dev) for x in c[:4]] for c in cases]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev) for _ in cases]
    torch.cuda.synchronize()
    for rep in range(3):   # the same four GEMMs, alternating streams, no host sync in between
        for i, (c, t) in enumerate(zip(cases, dev_cases)):
            with torch.cuda.stream(streams[i % 2]):
                bh.nvfp4_bf16_gemm(M, N, K, *t, outs[i], c[4])
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    for c, o in zip(cases, outs):
        _check(M, N, K, c, o.view(torch.int16))


def test_calls_from_several_host_threads():
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    work = []
    for M, N, K in SHAPES:
        for c in _cases(M, N, K, 2, 500):
            work.append((M, N, K, c, [torch.from_numpy(x).to(dev) for x in c[:4]],
                         torch.empty((M, N), dtype=torch.bfloat16, device=dev)))
    torch.cuda.synchronize()

    def run(items, errors):
        try:
            s = torch.cuda.Stream(device=dev)
            with torch.cuda.stream(s):
                for _ in range(4):
                    for M, N, K, c, t, out in items:
                        bh.nvfp4_bf16_gemm(M, N, K, *t, out, c[4])
            s.synchronize()
        except Exception as e:   # reported on the main thread
            errors.append(repr(e))

    for trial in range(2):
        errors = []
        for _, _, _, _, _, out in work:
            out.fill_(float("nan"))
        torch.cuda.synchronize()
        threads = [threading.Thread(target=run, args=(work[i::3], errors)) for i in range(3)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
        assert not errors, f"trial {trial}: {errors}"
        torch.cuda.synchronize()
        assert bh.device_status(0) == 0
        for M, N, K, c, _, out in work:
            _check(M, N, K, c, out.view(torch.int16))
