"""Stream order of the skinny schedule under programmatic dependent launch (M <= 128).

The skinny kernel sets up and prefetches its first B / SFB tiles into L2 while the kernel
launched just before it on the same stream is finishing; every load, store and workspace
access waits for that kernel to complete.  These tests launch GEMMs back to back without host
synchronisation and check that the results are bit-identical to the schedule without the
prefetch ("skinny_noprefetch") and to the oracle, including the cases where the previous
kernel wrote the very bytes the next GEMM reads as B (a device quantiser, or the previous
GEMM's output)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


def _dev_operands(M, N, K, seed, std_b=0.02):
    import torch

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=seed, std_b=std_b)
    dev = torch.device("cuda:0")
    return (A, SFA, B, SFB, alpha), tuple(torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))


def _bits(t):
    import torch

    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_back_to_back_rotating_weights_match_no_prefetch():
    import torch
    import blackhole_b200 as bh

    M, N, K = 16, 4096, 2048
    sets = [_dev_operands(M, N, K, seed=300 + i) for i in range(3)]
    ref = []
    for host, (tA, tSFA, tB, tSFB) in sets:
        D = torch.empty((M, N), dtype=torch.bfloat16, device="cuda:0")
        bh.nvfp4_bf16_gemm_ex(M, N, K, tA, tSFA, tB, tSFB, D, host[4], schedule="skinny_noprefetch")
        torch.cuda.synchronize()
        ref.append(_bits(D))
    outs = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda:0") for _ in range(12)]
    for i, D in enumerate(outs):  # no synchronisation between launches
        host, (tA, tSFA, tB, tSFB) = sets[i % 3]
        bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, host[4])
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    for i, D in enumerate(outs):
        assert np.array_equal(_bits(D), ref[i % 3]), f"launch {i} differs from the schedule without prefetch"
    host = sets[0][0]
    (bad, maxerr, ratio, _), _ = C.check_full(M, N, K, *host, ref[0])
    assert bad == 0, f"{bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"


def test_weights_quantized_just_before_the_gemm():
    """The device quantiser rewrites one weight buffer before every GEMM, with no sync."""
    import torch
    import blackhole_b200 as bh

    M, N, K = 16, 2048, 2048
    rng = np.random.default_rng(7)
    A, SFA, gA = O.quantize(O.gen_normal(41, M * K).reshape(M, K))
    dev = torch.device("cuda:0")
    tA, tSFA = torch.from_numpy(A).to(dev), torch.from_numpy(SFA).to(dev)
    tB = torch.empty(N * K // 2, dtype=torch.uint8, device=dev)
    tSFB = torch.empty(bh.sf_storage_bytes(N, K), dtype=torch.uint8, device=dev)
    scales = torch.empty(2, dtype=torch.float32, device=dev)
    xs = [rng.standard_normal((N, K), dtype=np.float32) * (0.5 + i) for i in range(4)]
    host_q = [O.quantize(x) for x in xs]  # (packed, sf, g), bit-exact with the device quantiser
    alphas = [float(np.float32(gA) * np.float32(g)) for _, _, g in host_q]
    tXs = [torch.from_numpy(x).to(dev) for x in xs]
    torch.cuda.synchronize()  # the uploads are not what is being tested
    outs = []
    for i, tX in enumerate(tXs):
        bh.nvfp4_quantize(tX, N, K, tB, tSFB, scales)
        D = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alphas[i])
        outs.append(D)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    for i, D in enumerate(outs):
        packed, sf, _ = host_q[i]
        (bad, maxerr, ratio, _), _ = C.check_full(M, N, K, A, SFA, packed, sf, alphas[i], _bits(D))
        assert bad == 0, f"gemm {i}: {bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"


def test_weights_aliasing_previous_gemm_output_are_read_in_order():
    """GEMM 2 reads, as its packed B, the bytes GEMM 1 has just written as D."""
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    (h1, (a1, sfa1, b1, sfb1)) = _dev_operands(256, 2048, 1024, seed=51, std_b=1.0)
    M2, N2, K2 = 16, 1024, 1024
    (h2, (a2, sfa2, _, sfb2)) = _dev_operands(M2, N2, K2, seed=52)
    results = []
    for schedule in ("skinny_noprefetch", "auto"):
        D1 = torch.full((256, 2048), -1, dtype=torch.int16, device=dev)  # stale bytes: 0xFF
        torch.cuda.synchronize()
        bh.nvfp4_bf16_gemm(256, 2048, 1024, a1, sfa1, b1, sfb1, D1, h1[4])
        b2 = D1.view(torch.uint8).reshape(-1)[: N2 * K2 // 2]
        D2 = torch.empty((M2, N2), dtype=torch.bfloat16, device=dev)
        bh.nvfp4_bf16_gemm_ex(M2, N2, K2, a2, sfa2, b2, sfb2, D2, h2[4], schedule=schedule)
        torch.cuda.synchronize()
        results.append((_bits(D2), b2.cpu().numpy().copy()))
    assert bh.device_status(0) == 0
    (np_bits, np_b2), (auto_bits, auto_b2) = results
    assert np.array_equal(np_b2, auto_b2)
    assert np.array_equal(np_bits, auto_bits)
    ref, absdot = O.gemm_full(M2, N2, K2, h2[0], h2[1], auto_b2, h2[3], h2[4])
    bad, maxerr, ratio, _ = O.check(ref, auto_bits, h2[4], K2, absdot)
    assert bad == 0, f"{bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"
