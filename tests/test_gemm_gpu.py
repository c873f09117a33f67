"""GPU parity of the sm_100a NVFP4 GEMM against the CPU oracle, through the C ABI.

Tolerance (per element): |got - ref| <= ulp_bf16(max(|ref|,|got|)) + |alpha|*K*2^-24*sum_k|a_k b_k|,
i.e. one BF16 ulp of the output plus the worst-case FP32 reassociation error of the K-term
sum; the per-term products are exact in FP32.  The reference example's own check
(rel <= 0.05, example/nvfp4_bf16_gemm.cu:169-172) is asserted as well."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _gold(name):
    man = json.load(open(os.path.join(GOLD, "manifest.json")))
    dt = {"uint8": np.uint8, "uint16": np.uint16}[man[name]["dtype"]]
    return np.fromfile(os.path.join(GOLD, name), dtype=dt)


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (256, 384, 512)])
def test_reference_example_fixtures_bit_exact(M, N, K):
    """Inputs drawn like the reference example; every partial sum is exact in FP32, so the
    GPU must reproduce the example's host loop bit for bit."""
    p = f"gemm_{M}x{N}x{K}_"
    A, SFA, B, SFB, D = (_gold(p + s) for s in ("A.u8", "SFA.u8", "B.u8", "SFB.u8", "D.u16"))
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, 1.0)
    assert np.array_equal(got.ravel(), D)


def test_config0_full_1024_cubed():
    M = N = K = 1024
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=0)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} elements outside tolerance (max err {maxerr}, max err/tol {ratio})"
    assert rel <= 0.05


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 256),      # one tile, one k-tile
    (128, 128, 512),      # N % 256 == 128: half of the B box is out of range
    (200, 384, 768),      # ragged M, ragged N tile, 3 k-tiles
    (1, 256, 1024),       # decode M=1
    (16, 1024, 2048),     # decode M=16
    (64, 512, 4096),
    (384, 640, 256),
    (130, 128, 8192),     # long K
])
def test_shapes_full(M, N, K):
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M * 7 + N, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, maxerr, ratio, rel), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


def test_alpha_scales_output():
    M, N, K = 128, 256, 512
    A, SFA, B, SFB, _ = C.make_operands(M, N, K, seed=11)
    for alpha in (1.0, 0.5, -3.25, 1e-3):
        got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
        (bad, *_), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
        assert bad == 0


@pytest.mark.parametrize("schedule,M,N,K", [("skinny", 16, 1024, 512), ("1sm", 128, 512, 512),
                                            ("2sm", 512, 512, 512)])
def test_alpha_edge_values(schedule, M, N, K):
    """alpha = +-0 (signed zeros out); +-1e32 (alpha * acc straddles the top of the BF16 range:
    most results round to +-inf, the rest stay finite); 3e37 (alpha * acc overflows FP32);
    1e-44 (an FP32 subnormal alpha: subnormal and zero BF16 results) through each schedule's
    epilogue.  Zeros and infinities must match the oracle bit for bit, finite values the usual
    tolerance."""
    A, SFA, B, SFB, _ = C.make_operands(M, N, K, seed=21 + M)
    for alpha in (0.0, -0.0, 1e32, -1e32, 3e37, 1e-44):
        got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule=schedule)
        ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
        rf, gf = O.bf16_bits_to_f32(ref.ravel()), O.bf16_bits_to_f32(got.ravel())
        special = ~np.isfinite(rf) | ~np.isfinite(gf) | (rf == 0) | (gf == 0)
        assert np.array_equal(got.ravel()[special], ref.ravel()[special]), f"alpha={alpha}"
        if abs(alpha) >= 1e32:
            assert np.isinf(rf).any(), "the case must reach the overflow"
        if alpha == 0.0:
            assert np.array_equal(got, ref), "signed zeros"
        fin = ~special
        bad, *_ = O.check(ref.ravel()[fin], got.ravel()[fin], alpha, K, ad.ravel()[fin])
        assert bad == 0, f"alpha={alpha}: {bad} finite elements outside tolerance"


@pytest.mark.parametrize("schedule,M,N,K", [("skinny", 16, 1024, 1024), ("1sm", 128, 512, 1024),
                                            ("2sm", 512, 512, 1024)])
def test_full_range_codes_and_scale_factors(schedule, M, N, K):
    """Every E2M1 code (signed zero included) and UE4M3 scale factors drawn from the whole
    finite range (codes 0..126: zero, 2^-9 .. 448), not the quantiser's narrow band: products
    span ~2^-20 .. 2^22, so the FP32 sums see large cancellations and rounding differences of
    order; the result must stay within the stated tolerance of the oracle."""
    rng = np.random.default_rng(1000 + M)
    A = rng.integers(0, 256, M * K // 2, dtype=np.uint8)
    B = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    SFA = np.zeros(O.sf_storage_bytes(M, K), dtype=np.uint8)
    SFB = np.zeros(O.sf_storage_bytes(N, K), dtype=np.uint8)
    SFA[O.sf_offsets(M, K).ravel()] = rng.integers(0, 127, M * (K // 16), dtype=np.uint8)
    SFB[O.sf_offsets(N, K).ravel()] = rng.integers(0, 127, N * (K // 16), dtype=np.uint8)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, 1.0, schedule=schedule)
    (bad, maxerr, ratio, _), ref = C.check_full(M, N, K, A, SFA, B, SFB, 1.0, got)
    assert bad == 0, f"{bad} elements outside tolerance (max err {maxerr}, err/tol {ratio})"
    assert np.isfinite(O.bf16_bits_to_f32(ref.ravel())).all()


@pytest.mark.parametrize("schedule,M,N,K", [("skinny", 16, 1024, 65536), ("1sm", 128, 512, 65536),
                                            ("2sm", 512, 512, 65536)])
def test_long_k(schedule, M, N, K):
    """K = 65536, past every config (configs[3] has K = 28672): 256 k-tiles of FP32 accumulation
    per output, and the K-dependent index arithmetic (k-tile coordinates, scale-factor atoms,
    stream-K units) at twice the configs' range; sampled against the oracle."""
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=77 + M, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, schedule=schedule)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got, S=2048)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


@pytest.mark.parametrize("schedule,M,N,K", [("skinny", 16, 1024, 2048), ("1sm", 128, 512, 1024),
                                            ("2sm", 512, 512, 1024)])
def test_operands_only_16_byte_aligned(schedule, M, N, K):
    """Callers pass slices of larger tensors: every operand (A, SFA, B, SFB, D) starts 16 bytes
    into a buffer, the least alignment the entry points accept, and no kernel may assume more."""
    import torch
    import blackhole_b200 as bh

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=88 + M, std_b=0.02)
    dev = torch.device("cuda:0")

    def at16(x):
        buf = torch.zeros(x.size + 64, dtype=torch.uint8, device=dev)
        view = buf[16:16 + x.size]
        view.copy_(torch.from_numpy(x.ravel()))
        assert view.data_ptr() % 128 == 16
        return view

    tA, tSFA, tB, tSFB = (at16(x) for x in (A, SFA, B, SFB))
    dbuf = torch.full((M * N + 32,), float("nan"), dtype=torch.bfloat16, device=dev)
    D = dbuf[8:8 + M * N]          # 16 bytes in
    assert D.data_ptr() % 128 == 16
    if schedule == "auto":
        bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha)
    else:
        bh.nvfp4_bf16_gemm_ex(M, N, K, tA, tSFA, tB, tSFB, D, alpha, schedule=schedule)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    got = D.view(torch.int16).cpu().numpy().view(np.uint16).reshape(M, N)
    ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    bad, maxerr, ratio, _ = O.check(ref, got, alpha, K, ad)
    assert bad == 0, f"{bad} elements outside tolerance (err/tol {ratio})"
    assert np.isnan(dbuf[:8].float().cpu().numpy()).all(), "wrote before D"
    assert np.isnan(dbuf[8 + M * N:].float().cpu().numpy()).all(), "wrote past D"


def test_outlier_activations_config3_style():
    M, N, K = 256, 512, 2048
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=3, std_b=0.02, outlier_p=0.01)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    (bad, *_), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0


def test_deterministic_across_runs():
    M, N, K = 256, 512, 1024
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=5)
    outs = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha, repeat=3)
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


@pytest.mark.parametrize("M", [1, 16, 64, 128])
def test_config2_decode_sampled(M):
    N, K = 28672, 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=2, std_b=0.02)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"


def test_config1_8192_cubed_sampled():
    M = N = K = 8192
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=1)
    got = C.run_gpu(M, N, K, A, SFA, B, SFB, alpha)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, A, SFA, B, SFB, alpha, got)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    assert rel <= 0.05
    assert not np.any(got == 0xFFFF), "unwritten output elements"


def _device_operands(M, N, K, seed_a, seed_b, std_b, outlier_p=0.0):
    """Operands built on the device the way bench.py builds them (torch generator + this
    library's quantiser, which is bit-exact with the oracle's), copied back for the oracle."""
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    ga = torch.Generator(device=dev)
    ga.manual_seed(seed_a)
    xa = torch.randn((M, K), generator=ga, device=dev)
    if outlier_p > 0:
        mask = torch.rand((M, K), generator=ga, device=dev) < outlier_p
        xa[mask] *= 20.0
        del mask
    gb = torch.Generator(device=dev)
    gb.manual_seed(seed_b)
    xb = torch.randn((N, K), generator=gb, device=dev) * std_b
    A, SFA, sa = bh.quantize_tensor(xa)
    B, SFB, sb = bh.quantize_tensor(xb)
    del xa, xb
    alpha = float(sa[1].item() * sb[1].item())
    return (A, SFA, B, SFB, alpha), tuple(t.cpu().numpy().reshape(-1) for t in (A, SFA, B, SFB))


def test_config3_prefill_outliers_full_size_sampled():
    """M=16384 N=8192 K=28672, 1% of the activations x20, weights N(0, 0.02^2)."""
    import torch
    import blackhole_b200 as bh

    M, N, K = 16384, 8192, 28672
    (A, SFA, B, SFB, alpha), host = _device_operands(M, N, K, 3, 3000, 0.02, outlier_p=0.01)
    D = torch.full((M, N), -1, dtype=torch.int16, device="cuda:0")
    bh.nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    got = D.cpu().numpy().view(np.uint16)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, *host, alpha, got, S=4096, seed=33)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    assert not np.any(got == 0xFFFF), "unwritten output elements"


def test_config4_shard_full_size_sampled():
    """configs[4] at P = 8: the per-GPU GEMM of one rank (M=32768, N=65536/8, K=8192)."""
    import torch
    import blackhole_b200 as bh

    M, N, K = 32768, 8192, 8192
    (A, SFA, B, SFB, alpha), host = _device_operands(M, N, K, 4, 4003, 1.0)
    D = torch.full((M, N), -1, dtype=torch.int16, device="cuda:0")
    bh.nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    got = D.cpu().numpy().view(np.uint16)
    bad, maxerr, ratio, rel = C.check_sampled(M, N, K, *host, alpha, got, S=4096, seed=44)
    assert bad == 0, f"{bad} bad (max err {maxerr}, err/tol {ratio})"
    assert not np.any(got == 0xFFFF), "unwritten output elements"
