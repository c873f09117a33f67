"""MXFP4 (OCP MX v1.0: E2M1 elements, one UE8M0 scale per 32 along K) through the C ABI.

The device quantiser must agree bit for bit with the oracle's (packed nibbles and every scale
byte, padding included), and each GEMM schedule must agree with the oracle's MXFP4 reference
GEMM within the same per-element tolerance as the NVFP4 path, on aligned, ragged-N and K-tail
shapes."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed, std_a=1.0, std_b=1.0):
    xa = O.gen_normal(seed, M * K, 0.0, std_a).reshape(M, K)
    xb = O.gen_normal(seed + 1000003, N * K, 0.0, std_b).reshape(N, K)
    A, SFA = O.quantize_mxfp4(xa)
    B, SFB = O.quantize_mxfp4(xb)
    return A, SFA, B, SFB


def _run(M, N, K, A, SFA, B, SFB, alpha, schedule, repeat=1):
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    D = torch.full((M, N), -1, dtype=torch.int16, device=dev)  # NaN pattern: catches unwritten
    outs = []
    for _ in range(repeat):
        bh.mxfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha, schedule=schedule)
        torch.cuda.synchronize()
        outs.append(D.cpu().numpy().view(np.uint16).copy())
    assert bh.device_status(0) == 0
    return outs


def _check(M, N, K, schedule, seed, std_b=1.0, alpha=1.0, repeat=1):
    A, SFA, B, SFB = _operands(M, N, K, seed, std_b=std_b)
    outs = _run(M, N, K, A, SFA, B, SFB, alpha, schedule, repeat)
    ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha, fmt="mxfp4")
    for g in outs:
        bad, maxerr, ratio, _ = O.check(ref, g, alpha, K, ad)
        assert bad == 0, f"mxfp4 {schedule} {M}x{N}x{K}: {bad} bad (max err {maxerr}, err/tol {ratio})"
        assert not np.any(g == 0xFFFF)
    for g in outs[1:]:
        assert np.array_equal(g, outs[0]), "schedule is not deterministic"


@pytest.mark.parametrize("rows,K", [(1, 32), (128, 256), (200, 768), (130, 320), (16, 8192),
                                    (1000, 4096)])
@pytest.mark.parametrize("bf16", [False, True])
def test_device_quantiser_bit_exact(rows, K, bf16):
    import torch
    import blackhole_b200 as bh

    x = O.gen_normal(rows * 7 + K, rows * K, 0.0, 3.0).reshape(rows, K)
    # special blocks: all zero, subnormal-only, huge, and a mixed row of powers of two
    x[0, :32] = 0.0
    if K >= 64:
        x[0, 32:64] = np.float32(1e-40)
    if K >= 128:
        x[0, 64:96] = np.float32(3e38) * np.sign(x[0, 64:96])
        x[0, 96:128] = np.ldexp(np.float32(1.0), np.arange(-16, 16)).astype(np.float32)
    dev = torch.device("cuda:0")
    tX = torch.from_numpy(x).to(dev)
    if bf16:
        tX = tX.to(torch.bfloat16)
        x = tX.float().cpu().numpy()  # the oracle sees exactly the values the device reads
    packed_ref, sf_ref = O.quantize_mxfp4(x)
    packed = torch.full((rows, K // 2), 0xAA, dtype=torch.uint8, device=dev)
    sf = torch.full((bh.mxfp4_sf_storage_bytes(rows, K),), 0xAA, dtype=torch.uint8, device=dev)
    bh.mxfp4_quantize(tX, rows, K, packed, sf, x_is_bf16=bf16)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy().reshape(-1), packed_ref)
    assert np.array_equal(sf.cpu().numpy(), sf_ref)


def test_quantize_tensor_mxfp4_feeds_the_gemm():
    import torch
    import blackhole_b200 as bh

    M, N, K = 64, 1024, 2048
    dev = torch.device("cuda:0")
    xa = torch.from_numpy(O.gen_normal(5, M * K).reshape(M, K)).to(dev)
    xb = torch.from_numpy(O.gen_normal(6, N * K, 0.0, 0.05).reshape(N, K)).to(dev)
    A, SFA = bh.quantize_tensor_mxfp4(xa)
    B, SFB = bh.quantize_tensor_mxfp4(xb)
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bh.mxfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    hA, hSFA, hB, hSFB = (t.cpu().numpy().reshape(-1) for t in (A, SFA, B, SFB))
    ref, ad = O.gemm_full(M, N, K, hA, hSFA, hB, hSFB, 1.0, fmt="mxfp4")
    got = D.view(torch.int16).cpu().numpy().view(np.uint16)
    bad, maxerr, ratio, rel = O.check(ref, got, 1.0, K, ad)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    # and the quantised product stays close to the unquantised one
    exact = (xa @ xb.T).cpu().numpy()
    deq = O.bf16_bits_to_f32(got.ravel()).reshape(M, N)
    assert np.abs(deq - exact).max() < 0.25 * np.abs(exact).max()


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 768, 512), (1000, 1152, 768),
                                   (2048, 2048, 2048), (256, 1000, 512), (512, 512, 288),
                                   (384, 256, 416)])
def test_two_sm_schedule(M, N, K):
    _check(M, N, K, "2sm", seed=M + N + K)


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 640, 512), (300, 520, 512),
                                   (256, 384, 160)])
def test_one_sm_schedule(M, N, K):
    _check(M, N, K, "1sm", seed=M + 3 * N + K)


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (16, 4096, 8192), (64, 4096, 2048),
                                   (128, 1024, 4096), (16, 1000, 1024), (16, 1024, 96),
                                   (33, 520, 352)])
def test_skinny_schedule(M, N, K):
    _check(M, N, K, "skinny", seed=M * 11 + N, std_b=0.02, repeat=2)


@pytest.mark.parametrize("M,N,K,alpha", [(16, 2048, 4096, 0.5), (200, 1024, 1024, 1.0),
                                         (1024, 1024, 1024, 2.0)])
def test_auto_schedule_with_alpha(M, N, K, alpha):
    _check(M, N, K, "auto", seed=M + 7 * N, alpha=alpha)


def test_mxfp4_and_nvfp4_share_no_state():
    """Interleaved MXFP4 and NVFP4 GEMMs on the same buffers' shapes give each format's own
    result (the tensor-map cache keys include the scale-factor format)."""
    import torch
    import blackhole_b200 as bh
    from tests import nvfp4_cases as C

    M, N, K = 256, 512, 1024
    dev = torch.device("cuda:0")
    mx = _operands(M, N, K, seed=77)
    nv = C.make_operands(M, N, K, seed=78)
    tmx = [torch.from_numpy(x).to(dev) for x in mx]
    tnv = [torch.from_numpy(x).to(dev) for x in nv[:4]]
    Dm = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    Dn = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    for _ in range(2):
        bh.mxfp4_bf16_gemm(M, N, K, tmx[0], tmx[1], tmx[2], tmx[3], Dm)
        bh.nvfp4_bf16_gemm(M, N, K, tnv[0], tnv[1], tnv[2], tnv[3], Dn, nv[4])
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    ref_m, ad_m = O.gemm_full(M, N, K, *mx, 1.0, fmt="mxfp4")
    ref_n, ad_n = O.gemm_full(M, N, K, *nv[:4], nv[4])
    got_m = Dm.view(torch.int16).cpu().numpy().view(np.uint16)
    got_n = Dn.view(torch.int16).cpu().numpy().view(np.uint16)
    assert O.check(ref_m, got_m, 1.0, K, ad_m)[0] == 0
    assert O.check(ref_n, got_n, nv[4], K, ad_n)[0] == 0
