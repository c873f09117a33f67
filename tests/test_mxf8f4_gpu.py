"""MXFP8 x MXFP4 (E4M3 activations x E2M1 weights, UE8M0 scales per 32) through the C ABI.

The device MXFP8 quantiser must agree bit for bit with the oracle's, and every schedule of
the tcgen05 kind::mxf8f6f4 GEMM (the E2M1 operand expanded to a byte per element by the TMA
unit) must agree with the oracle's mixed-format reference GEMM within the NVFP4 path's
per-element tolerance, on aligned, ragged-N and K = 128 * odd shapes."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed, std_a=1.0, std_b=1.0):
    xa = O.gen_normal(seed, M * K, 0.0, std_a).reshape(M, K)
    xb = O.gen_normal(seed + 1000003, N * K, 0.0, std_b).reshape(N, K)
    A, SFA = O.quantize_mxfp8(xa)
    B, SFB = O.quantize_mxfp4(xb)
    return A, SFA, B, SFB


def _check(M, N, K, schedule, seed, std_b=1.0, alpha=1.0, repeat=1):
    import torch
    import blackhole_b200 as bh

    A, SFA, B, SFB = _operands(M, N, K, seed, std_b=std_b)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    D = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    outs = []
    for _ in range(repeat):
        bh.mxf8f4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha, schedule=schedule)
        torch.cuda.synchronize()
        outs.append(D.cpu().numpy().view(np.uint16).copy())
    assert bh.device_status(0) == 0
    ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha, fmt="mxf8f4")
    for g in outs:
        bad, maxerr, ratio, _ = O.check(ref, g, alpha, K, ad)
        assert bad == 0, f"mxf8f4 {schedule} {M}x{N}x{K}: {bad} bad (max err {maxerr}, err/tol {ratio})"
        assert not np.any(g == 0xFFFF)
    for g in outs[1:]:
        assert np.array_equal(g, outs[0]), "schedule is not deterministic"


@pytest.mark.parametrize("rows,K", [(1, 32), (128, 256), (200, 768), (130, 320), (16, 8192)])
@pytest.mark.parametrize("bf16", [False, True])
def test_device_mxfp8_quantiser_bit_exact(rows, K, bf16):
    import torch
    import blackhole_b200 as bh

    x = O.gen_normal(rows * 5 + K, rows * K, 0.0, 7.0).reshape(rows, K)
    x[0, :32] = 0.0
    if K >= 64:
        x[0, 32:64] = np.float32(1e-40)                     # subnormal-only block
    if K >= 128:
        x[0, 64:96] = np.float32(1.9 * 2.0 ** 8)            # scaled past 448: saturates
        x[0, 96:128] = np.ldexp(np.float32(1.0), np.arange(-16, 16)).astype(np.float32)
    dev = torch.device("cuda:0")
    tX = torch.from_numpy(x).to(dev)
    if bf16:
        tX = tX.to(torch.bfloat16)
        x = tX.float().cpu().numpy()
    q_ref, sf_ref = O.quantize_mxfp8(x)
    q = torch.full((rows, K), 0xAA, dtype=torch.uint8, device=dev)
    sf = torch.full((bh.mxfp4_sf_storage_bytes(rows, K),), 0xAA, dtype=torch.uint8, device=dev)
    bh.mxfp8_quantize(tX, rows, K, q, sf, x_is_bf16=bf16)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(-1), q_ref)
    assert np.array_equal(sf.cpu().numpy(), sf_ref)


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (512, 768, 512), (1000, 1152, 768),
                                   (2048, 2048, 2048), (256, 1000, 384), (384, 256, 640)])
def test_two_sm_schedule(M, N, K):
    _check(M, N, K, "2sm", seed=M + N + K)


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 640, 512), (300, 520, 384)])
def test_one_sm_schedule(M, N, K):
    _check(M, N, K, "1sm", seed=M + 3 * N + K)


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (16, 4096, 8192), (64, 4096, 2048),
                                   (128, 1024, 4096), (16, 1000, 1024), (33, 520, 384)])
def test_skinny_schedule(M, N, K):
    _check(M, N, K, "skinny", seed=M * 11 + N, std_b=0.02, repeat=2)


@pytest.mark.parametrize("M,N,K,alpha", [(16, 2048, 4096, 0.5), (1024, 1024, 1024, 2.0)])
def test_auto_schedule_with_alpha(M, N, K, alpha):
    _check(M, N, K, "auto", seed=M + 7 * N, alpha=alpha)


def test_quantised_on_device_end_to_end():
    import torch
    import blackhole_b200 as bh

    M, N, K = 64, 1024, 2048
    dev = torch.device("cuda:0")
    xa = torch.from_numpy(O.gen_normal(5, M * K).reshape(M, K)).to(dev)
    xb = torch.from_numpy(O.gen_normal(6, N * K, 0.0, 0.05).reshape(N, K)).to(dev)
    A, SFA = bh.quantize_tensor_mxfp8(xa)
    B, SFB = bh.quantize_tensor_mxfp4(xb)
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bh.mxf8f4_bf16_gemm(M, N, K, A, SFA, B, SFB, D)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    hA, hSFA, hB, hSFB = (t.cpu().numpy().reshape(-1) for t in (A, SFA, B, SFB))
    ref, ad = O.gemm_full(M, N, K, hA, hSFA, hB, hSFB, 1.0, fmt="mxf8f4")
    got = D.view(torch.int16).cpu().numpy().view(np.uint16)
    assert O.check(ref, got, 1.0, K, ad)[0] == 0
    exact = (xa @ xb.T).cpu().numpy()
    deq = O.bf16_bits_to_f32(got.ravel()).reshape(M, N)
    assert np.abs(deq - exact).max() < 0.25 * np.abs(exact).max()
